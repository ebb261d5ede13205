// Internal launch interface shared by the kernel translation units and the C-ABI layer.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>

namespace qkv {

// Tensor-core (tcgen05) path for multi-token attention over the quantized cache: head_dim
// 128, GQA dividing 128, no mask or causal, one length for every batch row.
struct TcPlan {
  int tokens_per_tile;  // query tokens of one GQA group in a 128-row MMA tile
  int tiles;            // 128-row tiles per CTA (1 or 2)
  int tblocks;          // CTAs along the query tokens
  int splits;           // CTAs along the keys
  int chunk;            // keys per split (multiple of the 128-key tile)
  int parts;            // partial rows per output row (= splits)
  int parts_bound;      // parts at the requested split count, >= parts; unlike parts (whose
                        // chunk rounding can lower it) it never decreases as n grows
};

// Everything one attention launch needs (device pointers; sizes already validated).
struct AttnArgs {
  const void* q;
  const void* kw;
  const void* ks;
  const void* kb;
  const void* vw;
  const void* vs;
  const void* vb;
  void* out;
  int B, HQ, HKV, S, D, NP;
  int n;                 // key count when lens == nullptr
  const int* lens;       // device int32[B] or nullptr
  const int* pos_base;   // device int32[B] or nullptr
  const int* total_lens; // device int32[B] or nullptr
  int bits;
  int dtype;  // QKV_BF16 / QKV_F16 (q, out, scales, biases, additive mask)
  float scale;
  int mask_kind;
  const void* mask;
  int mask_nk;
  long long mask_sb, mask_sh, mask_sq;
  int out_kind;
  int splits;   // resolved split count (>= 1)
  int chunk;    // keys per split (multiple of the 16-key warp tile)
  int balanced; // > 0 (ragged lens, merged in-kernel): the splits CTAs of a (kv head, row
                // group) are shared by the batches by key count, chunk = total / balanced
  void* workspace;
  size_t ws_bytes;
  int* status;  // device status word for bounded-wait failures
  int prefetch_limit;  // cache positions below this may be read before the kernel that
                       // precedes this one in the stream has finished (see qkv_decode.cu)
  const void* k_new;   // decode path only: the S new tokens' K and V (B, HKV, S, D) in dtype,
  const void* v_new;   // quantized into the cache at [new_pos, new_pos + S) by the attention
  int new_pos;         // kernel itself before it reads them (nullptr: already in the cache)
  bool use_tc;         // multi-token tensor-core path (qkv_prefill_tc.cu) instead of decode
  TcPlan tc;
  int phantom;                 // test hook (qkv_test_hooks): extra partial sets to wait for
  unsigned long long spin_ns;  // test hook: merge polling bound (0 = the library default)
};

// Values set by qkv_test_hooks (0 = off / library default).
struct TestHooks {
  int phantom_splits;
  long long spin_ns;
};
TestHooks test_hooks();

// Split-KV decode/verify path (mma.sync, keys as MMA rows, query rows as columns).
// The attention workspace holds partial rows whose words read 0 until written; it is zero
// before the first call and every call leaves it zero (the readers clear what they read).
int decode_rows_per_group(int R, int D);    // query rows handled by one CTA (8 or 16)
size_t decode_workspace_bytes(int B, int HQ, int S, int D, int splits);
void decode_plan(int B, int HQ, int HKV, int S, int D, int bits, int n_max, int want_splits,
                 int* splits, int* chunk);
// Ragged batches merged in-kernel: CTAs per (kv head, row group) shared by the batches
// (= balanced + B); returns balanced. The workspace need is decode_balanced_bytes.
int decode_plan_balanced(int B, int HQ, int HKV, int S, int D, int bits);
size_t decode_balanced_bytes(int B, int HQ, int S, int D, int balanced);
// resident CTAs per SM the decode kernel is built for (register budget per instantiation)
inline int decode_ctas_per_sm(int R, int D, int bits) {
  return (R <= 8 && D <= 128 && bits == 8) ? 3 : 2;
}

// Decode/verify attention: one launch whose last splits merge the partials, or (a grid too
// large to be resident at once) the split kernel's plain partial rows + combine_kernel.
int launch_decode(const AttnArgs& a, cudaStream_t st);
bool decode_merges_in_kernel(const AttnArgs& a);
// workspace of the two-launch route: plain partial rows [splits][B*HQ*S][D+4]
size_t decode_fallback_bytes(int B, int HQ, int S, int D, int splits);
int launch_split_only(const AttnArgs& a, cudaStream_t st);  // partial rows into a.workspace

// clear: the partials are in an attention workspace; zero every word read
int launch_combine(const float* parts, int n_parts, long long part_stride_rows, long long rows,
                   int D, void* out, int out_dtype, int out_kind, cudaStream_t st,
                   bool clear = false);

// up to two tensors (K and V of one append) quantized by one launch
int launch_quantize_jobs(const void* const* x, int x_dtype, void* const* w, void* const* sc,
                         void* const* bi, int jobs, int B, int H, int S, int D, int NP,
                         int offset, int bits, int scale_dtype, cudaStream_t st);
int launch_quantize(const void* x, int x_dtype, void* w, void* sc, void* bi, int B, int H,
                    int S, int D, int NP, int offset, int bits, int scale_dtype,
                    cudaStream_t st);
int launch_dequantize(const void* w, const void* sc, const void* bi, void* out, long long rows,
                      int D, int bits, int dtype, int round_mode, cudaStream_t st);

int num_sms();

// Per-device caches in this library are indexed by device ordinal below this bound.
constexpr int kMaxDevices = 64;

// Zero the static scratch of qkv_attention_noalloc on the current device (enqueued on st);
// cudaSuccess without work when no call has resolved the scratch on this device yet.
cudaError_t noalloc_scratch_clear(cudaStream_t st);

// Byte-typed tiled tensor map over (RB, NP, bhs) packed codes; box (box_inner bytes,
// box_rows keys, 1), swizzled by the box's inner span. False if the driver refuses it.
bool make_code_map_bytes(CUtensorMap* m, const void* base, int RB, int NP, long long bhs,
                         int box_inner, int box_rows);


bool prefill_tc_eligible(int B, int HQ, int HKV, int S, int D, const int* lens,
                         const int* pos_base, const int* total_lens, int mask_kind);
TcPlan prefill_tc_plan(int B, int HQ, int HKV, int S, int n_max, int want_splits);
// Partial rows of every split (none when one split writes the normalized output directly).
size_t prefill_tc_workspace_bytes(int B, int HQ, int S, int D, const TcPlan& p, bool direct);
// combine = false leaves the split partials in a.workspace ([splits][B*HQ*S][D+4]).
int launch_prefill_tc(const AttnArgs& a, const TcPlan& p, bool combine, cudaStream_t st);

// Workspace bytes the last attention call on this thread asked for (set whenever its
// arguments were valid enough to plan the launch).
size_t last_workspace_need();

// Device address of the status word (qkv_device_status) on the current device; nullptr if
// it cannot be resolved.
int* device_status_word();

// Record a message for qkv_last_error() on this thread and return `code`.
int set_last_error(int code, const char* fmt, ...);

}  // namespace qkv
