// C-ABI entry points of libqkv.so: argument validation, kernel dispatch, error reporting.
// Every entry point returns a status and never aborts; kernels are only enqueued on the
// caller's stream (no allocation, no device synchronization) except qkv_device_status.
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include <algorithm>
#include <atomic>

#include "../../include/qkv.h"
#include "qkv_internal.h"


namespace qkv {

__device__ int g_device_status = 0;

namespace {
std::atomic<int> g_hook_phantom{0};
std::atomic<long long> g_hook_spin_ns{0};
}  // namespace

TestHooks test_hooks() { return TestHooks{g_hook_phantom.load(), g_hook_spin_ns.load()}; }

namespace {

thread_local char g_err[512] = "";
thread_local size_t g_last_need = 0;

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_check(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(QKV_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return QKV_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int* status_ptr() {
  // Address of the device status word on the current device, looked up once per device.
  static int* ptrs[kMaxDevices] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

int check_cache_shape(int D, int bits, int group_size) {
  if (bits != 4 && bits != 8) return fail(QKV_EUNSUPPORTED, "bits must be 4 or 8 (got %d)", bits);
  if (group_size != 64)
    return fail(QKV_EUNSUPPORTED, "group_size must be 64 (got %d)", group_size);
  if (D != 64 && D != 128 && D != 256)
    return fail(QKV_EUNSUPPORTED, "head_dim must be 64, 128 or 256 (got %d)", D);
  return QKV_OK;
}

}  // namespace

int num_sms() {
  static int cached[kMaxDevices] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) dev = 0;
  if (!cached[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
      v = 148;
    cached[dev] = v;
  }
  return cached[dev];
}

size_t last_workspace_need() { return g_last_need; }

int* device_status_word() { return status_ptr(); }

int set_last_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

}  // namespace qkv

using namespace qkv;

extern "C" {

int qkv_version(void) { return 100; }

const char* qkv_last_error(void) { return g_err; }

int qkv_device_status(void* stream, int reset) {
  int* p = status_ptr();
  if (!p) return fail(QKV_ECUDA, "device status word unavailable");
  int v = 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(&v, p, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return cuda_check("qkv_device_status");
  if (reset) {
    // The stream is synchronized: every kernel enqueued before this call has finished, so
    // no partial row can still land in the static scratch of qkv_attention_noalloc, which
    // is zeroed here (the merge reads a zero word as "not yet written"; a merge that gave up
    // may have left words behind).
    const int zero = 0;
    if (cudaMemcpyAsync(p, &zero, sizeof(int), cudaMemcpyHostToDevice, st) != cudaSuccess ||
        noalloc_scratch_clear(st) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess)
      return cuda_check("qkv_device_status reset");
  }
  return v;
}

int qkv_test_hooks(int phantom_splits, long long spin_ns) {
  if (phantom_splits < 0 || phantom_splits > 64 || spin_ns < 0)
    return fail(QKV_EINVAL, "bad test hook values (phantom %d, spin %lld ns)", phantom_splits,
                spin_ns);
  g_hook_phantom.store(phantom_splits);
  g_hook_spin_ns.store(spin_ns);
  return QKV_OK;
}

namespace {
int check_append(const void* x, int x_dtype, const void* w, const void* scales,
                 const void* biases, int B, int H, int S, int D, int NP, int offset, int bits,
                 int group_size, int scale_dtype) {
  int rc = check_cache_shape(D, bits, group_size);
  if (rc) return rc;
  if (!x || !w || !scales || !biases) return fail(QKV_EINVAL, "null pointer");
  if (B < 0 || H < 0 || S < 0 || offset < 0 || NP < 0)
    return fail(QKV_EINVAL, "negative size");
  if ((long long)offset + S > NP)
    return fail(QKV_EINVAL, "offset %d + S %d exceeds padded length %d", offset, S, NP);
  if (x_dtype != QKV_BF16 && x_dtype != QKV_F16 && x_dtype != QKV_F32)
    return fail(QKV_EINVAL, "bad x_dtype %d", x_dtype);
  if (scale_dtype != QKV_BF16 && scale_dtype != QKV_F16)
    return fail(QKV_EINVAL, "bad scale_dtype %d", scale_dtype);
  return QKV_OK;
}
}  // namespace

int qkv_quantize_append(const void* x, int x_dtype, void* w, void* scales, void* biases, int B,
                        int H, int S, int D, int NP, int offset, int bits, int group_size,
                        int scale_dtype, void* stream) {
  int rc = check_append(x, x_dtype, w, scales, biases, B, H, S, D, NP, offset, bits, group_size,
                        scale_dtype);
  if (rc) return rc;
  rc = launch_quantize(x, x_dtype, w, scales, biases, B, H, S, D, NP, offset, bits, scale_dtype,
                       static_cast<cudaStream_t>(stream));
  if (rc) return fail(rc, "quantize: unsupported shape");
  return cuda_check("qkv_quantize_append");
}

int qkv_quantize_append_kv(const void* k, const void* v, int x_dtype, void* kw, void* ks,
                           void* kb, void* vw, void* vs, void* vb, int B, int H, int S, int D,
                           int NP, int offset, int bits, int group_size, int scale_dtype,
                           void* stream) {
  int rc = check_append(k, x_dtype, kw, ks, kb, B, H, S, D, NP, offset, bits, group_size,
                        scale_dtype);
  if (rc) return rc;
  rc = check_append(v, x_dtype, vw, vs, vb, B, H, S, D, NP, offset, bits, group_size,
                    scale_dtype);
  if (rc) return rc;
  const void* xs[2] = {k, v};
  void* ws_[2] = {kw, vw};
  void* ss[2] = {ks, vs};
  void* bs[2] = {kb, vb};
  rc = launch_quantize_jobs(xs, x_dtype, ws_, ss, bs, 2, B, H, S, D, NP, offset, bits,
                            scale_dtype, static_cast<cudaStream_t>(stream));
  if (rc) return fail(rc, "quantize: unsupported shape");
  return cuda_check("qkv_quantize_append_kv");
}

int qkv_dequantize(const void* w, const void* scales, const void* biases, void* out,
                   long long rows, int D, int bits, int group_size, int dtype, int round_mode,
                   void* stream) {
  int rc = check_cache_shape(D, bits, group_size);
  if (rc) return rc;
  if (rows < 0) return fail(QKV_EINVAL, "negative rows");
  if (!w || !scales || !biases || !out) return fail(QKV_EINVAL, "null pointer");
  if (dtype != QKV_BF16 && dtype != QKV_F16) return fail(QKV_EINVAL, "bad dtype %d", dtype);
  if (round_mode != 0 && round_mode != 1) return fail(QKV_EINVAL, "bad round_mode %d", round_mode);
  rc = launch_dequantize(w, scales, biases, out, rows, D, bits, dtype, round_mode,
                         static_cast<cudaStream_t>(stream));
  if (rc) return fail(rc, "dequantize: unsupported shape");
  return cuda_check("qkv_dequantize");
}

size_t qkv_workspace_size(int B, int HQ, int HKV, int S, int D, int n_max, int bits,
                          int group_size) {
  (void)bits;
  (void)group_size;
  if (B <= 0 || HQ <= 0 || HKV <= 0 || S <= 0 || D <= 0 || HQ % HKV) return 0;
  int splits = 1, chunk = 16;
  decode_plan(B, HQ, HKV, S, D, bits, std::max(n_max, 1), 0, &splits, &chunk);
  size_t need = decode_workspace_bytes(B, HQ, S, D, splits);
  // ragged batches (per-batch lengths) share the CTAs by key count
  if (B > 1)
    need = std::max(need, decode_balanced_bytes(B, HQ, S, D,
                                                decode_plan_balanced(B, HQ, HKV, S, D, bits)));
  // multi-token calls may take the tensor-core path: room for its split partials too
  if (prefill_tc_eligible(B, HQ, HKV, S, D, nullptr, nullptr, nullptr, QKV_MASK_CAUSAL)) {
    // sized by the requested split count, so the answer never shrinks as n_max grows
    // (callers may size once for an upper bound of the key count)
    TcPlan tp = prefill_tc_plan(B, HQ, HKV, S, std::max(n_max, 1), 0);
    tp.parts = tp.parts_bound;
    need = std::max(need, prefill_tc_workspace_bytes(B, HQ, S, D, tp, false));
  }
  return need;
}

namespace {

// Validate and pack the shared arguments of qkv_attention / qkv_partials.
int setup_attn(AttnArgs& a, const void* q, const void* kw, const void* ks, const void* kb,
               const void* vw, const void* vs, const void* vb, void* out, int B, int HQ,
               int HKV, int S, int D, int NP, int n, const int* lens, const int* pos_base,
               const int* total_lens, int bits, int group_size, int dtype, float scale,
               int mask_kind, const void* mask, int mask_nk, long long mask_sb,
               long long mask_sh, long long mask_sq, int splits, void* workspace,
               size_t ws_bytes, bool direct, bool merge) {
  int rc = check_cache_shape(D, bits, group_size);
  if (rc) return rc;
  if (!q || !kw || !ks || !kb || !vw || !vs || !vb || !out)
    return fail(QKV_EINVAL, "null tensor pointer");
  if (B <= 0 || HQ <= 0 || HKV <= 0 || S <= 0 || NP <= 0 || n < 0)
    return fail(QKV_EINVAL, "bad sizes B=%d HQ=%d HKV=%d S=%d NP=%d n=%d", B, HQ, HKV, S, NP, n);
  if (HQ % HKV) return fail(QKV_EINVAL, "HQ %d is not a multiple of HKV %d", HQ, HKV);
  if (!lens && n > NP) return fail(QKV_EINVAL, "n %d exceeds padded length %d", n, NP);
  if (NP % 8) return fail(QKV_EALIGN, "padded length %d must be a multiple of 8", NP);
  if (!aligned16(q) || !aligned16(kw) || !aligned16(ks) || !aligned16(kb) || !aligned16(vw) ||
      !aligned16(vs) || !aligned16(vb) || !aligned16(out))
    return fail(QKV_EALIGN, "tensor pointers must be 16-byte aligned");
  if (dtype != QKV_BF16 && dtype != QKV_F16) return fail(QKV_EINVAL, "bad dtype %d", dtype);
  if (mask_kind < QKV_MASK_NONE || mask_kind > QKV_MASK_ADDITIVE)
    return fail(QKV_EINVAL, "bad mask kind %d", mask_kind);
  if ((mask_kind == QKV_MASK_BOOL || mask_kind == QKV_MASK_ADDITIVE) && (!mask || mask_nk <= 0))
    return fail(QKV_EINVAL, "mask array missing");
  if (splits < 0) return fail(QKV_EINVAL, "negative split count");

  a = AttnArgs{};
  a.q = q;
  a.kw = kw;
  a.ks = ks;
  a.kb = kb;
  a.vw = vw;
  a.vs = vs;
  a.vb = vb;
  a.out = out;
  a.B = B;
  a.HQ = HQ;
  a.HKV = HKV;
  a.S = S;
  a.D = D;
  a.NP = NP;
  a.n = lens ? std::min(n, NP) : n;
  a.lens = lens;
  a.pos_base = pos_base;
  a.total_lens = total_lens;
  a.bits = bits;
  a.dtype = dtype;
  a.scale = scale;
  // causal with one query token hides nothing: query S-1 sits at the last key
  a.mask_kind = (mask_kind == QKV_MASK_CAUSAL && S == 1 && !pos_base && !total_lens)
                    ? QKV_MASK_NONE
                    : mask_kind;
  a.mask = mask;
  a.mask_nk = mask_nk;
  a.mask_sb = mask_sb;
  a.mask_sh = mask_sh;
  a.mask_sq = mask_sq;
  a.status = status_ptr();
  // The kernel issued just before an attention call may be the append of its S tokens
  // (positions n-S..n-1); everything older is immutable during that kernel, so the attention
  // kernel may start streaming it early (programmatic dependent launch). With per-batch
  // lengths on the device nothing is read early.
  a.prefetch_limit = lens ? 0 : std::max(0, std::min(n, NP) - S);

  const int n_max = std::max(a.n, 1);
  const int R = (HQ / HKV) * S;
  const int rg = (R + decode_rows_per_group(R, D) - 1) / decode_rows_per_group(R, D);
  if ((long long)HKV * rg > 65535 || B > 65535)
    return fail(QKV_EUNSUPPORTED, "too many kv heads x query-row groups (%lld) or batch (%d)",
                (long long)HKV * rg, B);
  decode_plan(B, HQ, HKV, S, D, bits, n_max, splits, &a.splits, &a.chunk);
  size_t need = decode_workspace_bytes(B, HQ, S, D, a.splits);
  if (merge && lens && B > 1 && splits == 0) {
    // ragged batches: share the CTAs by key count instead of splitting every batch alike
    a.balanced = decode_plan_balanced(B, HQ, HKV, S, D, bits);
    a.splits = a.balanced + B;
    need = decode_balanced_bytes(B, HQ, S, D, a.balanced);
  }
  // (the tensor-core path's running max assumes a positive softmax scale)
  a.use_tc = prefill_tc_eligible(B, HQ, HKV, S, D, lens, pos_base, total_lens, a.mask_kind) &&
             scale > 0.f;
  if (a.use_tc) {
    a.tc = prefill_tc_plan(B, HQ, HKV, S, n_max, splits);
    need = prefill_tc_workspace_bytes(B, HQ, S, D, a.tc, direct);
  }
  if (merge && !a.use_tc) {
    const TestHooks h = test_hooks();
    if (!a.balanced && h.phantom_splits > 0) {
      a.phantom = h.phantom_splits;
      need = decode_workspace_bytes(B, HQ, S, D, a.splits + a.phantom);
    }
    a.spin_ns = (unsigned long long)h.spin_ns;
  }
  g_last_need = need;
  if (!workspace || ws_bytes < need)
    return fail(QKV_EWORKSPACE, "workspace %zu bytes < required %zu", ws_bytes, need);
  if (!aligned16(workspace)) return fail(QKV_EALIGN, "workspace must be 16-byte aligned");
  a.workspace = workspace;
  a.ws_bytes = ws_bytes;
  return QKV_OK;
}

}  // namespace

int qkv_attention(const void* q, const void* kw, const void* ks, const void* kb, const void* vw,
                  const void* vs, const void* vb, void* out, int B, int HQ, int HKV, int S, int D,
                  int NP, int n, const int* lens, const int* pos_base, const int* total_lens,
                  int bits, int group_size, int dtype, float scale, int mask_kind,
                  const void* mask, int mask_nk, long long mask_sb, long long mask_sh,
                  long long mask_sq, int out_kind, int splits, void* workspace, size_t ws_bytes,
                  void* stream) {
  if (out_kind != QKV_OUT_NORMALIZED && out_kind != QKV_OUT_PARTIAL)
    return fail(QKV_EINVAL, "bad out_kind %d", out_kind);
  AttnArgs a;
  int rc = setup_attn(a, q, kw, ks, kb, vw, vs, vb, out, B, HQ, HKV, S, D, NP, n, lens,
                      pos_base, total_lens, bits, group_size, dtype, scale, mask_kind, mask,
                      mask_nk, mask_sb, mask_sh, mask_sq, splits, workspace, ws_bytes,
                      out_kind == QKV_OUT_NORMALIZED, true);
  if (rc) return rc;
  a.out_kind = out_kind;
  rc = a.use_tc ? launch_prefill_tc(a, a.tc, true, static_cast<cudaStream_t>(stream))
                : launch_decode(a, static_cast<cudaStream_t>(stream));
  if (rc) return fail(rc, "attention: unsupported configuration");
  return cuda_check("qkv_attention");
}

int qkv_partials(const void* q, const void* kw, const void* ks, const void* kb, const void* vw,
                 const void* vs, const void* vb, float* parts, size_t parts_bytes, int* n_parts,
                 int B, int HQ, int HKV, int S, int D, int NP, int n, const int* lens,
                 const int* pos_base, const int* total_lens, int bits, int group_size,
                 int dtype, float scale, int mask_kind, const void* mask, int mask_nk,
                 long long mask_sb, long long mask_sh, long long mask_sq, int splits,
                 void* stream) {
  if (!n_parts) return fail(QKV_EINVAL, "n_parts is null");
  AttnArgs a;
  int rc = setup_attn(a, q, kw, ks, kb, vw, vs, vb, parts, B, HQ, HKV, S, D, NP, n, lens,
                      pos_base, total_lens, bits, group_size, dtype, scale, mask_kind, mask,
                      mask_nk, mask_sb, mask_sh, mask_sq, splits, parts, parts_bytes, false,
                      false);
  if (rc) return rc;
  a.out_kind = QKV_OUT_PARTIAL;
  *n_parts = a.use_tc ? a.tc.parts : a.splits;
  rc = a.use_tc ? launch_prefill_tc(a, a.tc, false, static_cast<cudaStream_t>(stream))
                : launch_split_only(a, static_cast<cudaStream_t>(stream));
  if (rc) return fail(rc, "partials: unsupported configuration");
  return cuda_check("qkv_partials");
}

int qkv_combine(const float* parts, int n_parts, long long rows, int D, void* out, int out_dtype,
                int out_kind, void* stream) {
  if (!parts || !out) return fail(QKV_EINVAL, "null pointer");
  if (n_parts <= 0 || rows < 0) return fail(QKV_EINVAL, "bad sizes");
  if (D != 64 && D != 128 && D != 256) return fail(QKV_EUNSUPPORTED, "head_dim %d", D);
  if (out_dtype != QKV_BF16 && out_dtype != QKV_F16) return fail(QKV_EINVAL, "bad dtype");
  if (out_kind != QKV_OUT_NORMALIZED && out_kind != QKV_OUT_PARTIAL)
    return fail(QKV_EINVAL, "bad out_kind %d", out_kind);
  const int rc =
      launch_combine(parts, n_parts, rows, rows, D, out, out_dtype, out_kind,
                     static_cast<cudaStream_t>(stream));
  if (rc) return fail(rc, "combine: unsupported");
  return cuda_check("qkv_combine");
}

int qkv_prefill(const void* q, const void* k_new, const void* v_new, void* kw, void* ks, void* kb,
                void* vw, void* vs, void* vb, void* out, int B, int HQ, int HKV, int S, int D,
                int NP, int offset, int bits, int group_size, int dtype, float scale,
                void* workspace, size_t ws_bytes, void* stream) {
  if (!k_new || !v_new) return fail(QKV_EINVAL, "null new-token K/V");
  int rc = check_append(k_new, dtype, kw, ks, kb, B, HKV, S, D, NP, offset, bits, group_size,
                        dtype);
  if (rc) return rc;
  rc = check_append(v_new, dtype, vw, vs, vb, B, HKV, S, D, NP, offset, bits, group_size, dtype);
  if (rc) return rc;
  AttnArgs a;
  rc = setup_attn(a, q, kw, ks, kb, vw, vs, vb, out, B, HQ, HKV, S, D, NP, offset + S, nullptr,
                  nullptr, nullptr, bits, group_size, dtype, scale, QKV_MASK_CAUSAL, nullptr, 0,
                  0, 0, 0, 0, workspace, ws_bytes, true, true);
  if (rc) return rc;
  a.out_kind = QKV_OUT_NORMALIZED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int R = (HQ / HKV) * S;
  if (!a.use_tc && R <= decode_rows_per_group(R, D)) {
    // one query-row group per kv head (a decode step, or a short draft block at small GQA):
    // the attention kernel quantizes the new tokens into the cache itself, one launch
    a.k_new = k_new;
    a.v_new = v_new;
    a.new_pos = offset;
    rc = launch_decode(a, st);
  } else {
    // K and V of the new tokens in one launch, then attention
    const void* xs[2] = {k_new, v_new};
    void* ws_[2] = {kw, vw};
    void* ss[2] = {ks, vs};
    void* bs[2] = {kb, vb};
    rc = launch_quantize_jobs(xs, dtype, ws_, ss, bs, 2, B, HKV, S, D, NP, offset, bits, dtype,
                              st);
    if (rc) return fail(rc, "quantize: unsupported shape");
    rc = a.use_tc ? launch_prefill_tc(a, a.tc, true, st) : launch_decode(a, st);
  }
  if (rc) return fail(rc, "prefill: unsupported configuration");
  return cuda_check("qkv_prefill");
}

}  // extern "C"
