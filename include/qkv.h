/*
 * qkv.h — C ABI of chad_b200's quantized-KV attention library (libqkv.so).
 *
 * The library replaces the quantized-KV attention path of nathansutton/chad
 * (src/chad/mlx_qsdpa.py) on NVIDIA B200 (sm_100a). bf16/fp16 queries attend over an
 * MLX-layout affine-quantized KV cache:
 *
 *   codes   uint32  (B, H, NP, D*bits/32)   4- or 8-bit codes packed LSB-first
 *   scales  T       (B, H, NP, D/64)        per group of 64 along head_dim
 *   biases  T       (B, H, NP, D/64)
 *
 * with T the query dtype (bf16 or fp16), exactly the (w, scales, biases) tuples that
 * mlx-lm's QuantizedKVCache hands to the reference (mlx_qsdpa.py:575-576, 646-656).
 * NP is the padded allocation length; only the first `n` (or lens[b]) positions are read
 * as keys, so anything in the padded tail is ignored (tests/test_mlx_qsdpa.py:82-95).
 *
 * Conventions for every entry point:
 *   - all pointers are device pointers owned by the caller; nothing is allocated or freed;
 *   - work is enqueued on `stream` (a cudaStream_t; NULL = legacy default stream) and the
 *     call never synchronizes the device, so calls on one stream are reentrant;
 *   - the return value is a status: QKV_OK (0) or a negative QKV_E* code, never an abort;
 *     qkv_last_error() returns a human-readable message for the calling thread;
 *   - shapes use int, element strides long long; pointers must be 16-byte aligned;
 *   - per-device state (symbol addresses, SM counts, occupancy) is looked up once per device
 *     and kept for the life of the process: after cudaDeviceReset, restart the process.
 */
#ifndef CHAD_B200_QKV_H
#define CHAD_B200_QKV_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define QKV_OK 0
#define QKV_EINVAL (-1)       /* invalid argument or shape */
#define QKV_EUNSUPPORTED (-2) /* valid but not implemented (e.g. head_dim 96) */
#define QKV_ECUDA (-3)        /* CUDA launch/runtime error; see qkv_last_error() */
#define QKV_EWORKSPACE (-4)   /* workspace missing or smaller than qkv_workspace_size() */
#define QKV_EALIGN (-5)       /* pointer or padded length breaks the alignment contract */
#define QKV_EDEVICE (-6)      /* a kernel gave up on a bounded wait (see qkv_device_status) */

/* element types */
#define QKV_BF16 0
#define QKV_F16 1
#define QKV_F32 2

/* mask kinds */
#define QKV_MASK_NONE 0
#define QKV_MASK_CAUSAL 1   /* query s of S sits at position total_len - S + s */
#define QKV_MASK_BOOL 2     /* uint8 keep-mask (1 = attend), (B,HQ,S,mask_nk) by strides */
#define QKV_MASK_ADDITIVE 3 /* additive mask in the query dtype, same indexing */

/* output kinds of qkv_attention */
#define QKV_OUT_NORMALIZED 0 /* out: (B,HQ,S,D) in the query dtype */
#define QKV_OUT_PARTIAL 1    /* out: float (B,HQ,S,D+4) rows of [O(D), m, l, 0, 0] */

/* Library version (major*10000 + minor*100 + patch). */
int qkv_version(void);

/* Message for the last non-zero status returned on the calling thread. */
const char* qkv_last_error(void);

/* Device-side status word: 0, or a QKV_EDEVICE code left by a kernel whose bounded
 * wait ran out (every wait in the library gives up after about 2 s instead of hanging).
 * Synchronizes `stream`. reset != 0 then clears the word and zeroes the static scratch of
 * qkv_attention_noalloc on the current device (a merge that gave up may have left words
 * behind). A caller-owned attention workspace is the caller's to zero again after a
 * non-zero status. No counterpart in the reference (MLX kernels have no bounded waits). */
int qkv_device_status(void* stream, int reset);

/* Testing hooks (no counterpart in the reference), process-wide, 0 = off:
 *   phantom_splits: decode merges wait for this many extra partial sets that no CTA
 *                   writes, so their bounded wait runs out (the workspace must hold them);
 *   spin_ns:        bound on that wait in nanoseconds instead of the default 2 s.
 * Lets a test drive the timeout path (QKV_EDEVICE status, recovery) without a GPU fault. */
int qkv_test_hooks(int phantom_splits, long long spin_ns);

/*
 * Quantize S new rows per (b,h) and write them into the padded cache at positions
 * [offset, offset+S): the quantize step of mlx-lm QuantizedKVCache.update_and_fetch
 * (exercised at tests/test_mlx_qsdpa.py:45-49; cache built at src/chad/engine.py:546-548).
 *   x:      (B, H, S, D) in x_dtype (QKV_BF16 / QKV_F16 / QKV_F32), contiguous
 *   w:      uint32 (B, H, NP, D*bits/32); scales/biases (B, H, NP, D/group_size)
 *           in scale_dtype (QKV_BF16 / QKV_F16)
 * Requires offset + S <= NP and group_size == 64.
 */
int qkv_quantize_append(const void* x, int x_dtype, void* w, void* scales, void* biases,
                        int B, int H, int S, int D, int NP, int offset, int bits,
                        int group_size, int scale_dtype, void* stream);

/*
 * K and V of the same S new rows in one launch: qkv_quantize_append on (k, kw, ks, kb) and
 * on (v, vw, vs, vb), as mlx-lm's QuantizedKVCache.update_and_fetch quantizes both per call
 * (tests/test_mlx_qsdpa.py:45-49). Same argument rules; k and v share x_dtype and shape.
 */
int qkv_quantize_append_kv(const void* k, const void* v, int x_dtype, void* kw, void* ks,
                           void* kb, void* vw, void* vs, void* vb, int B, int H, int S, int D,
                           int NP, int offset, int bits, int group_size, int scale_dtype,
                           void* stream);

/*
 * Dequantize `rows` packed rows of D values: the semantics of mx.dequantize as called at
 * src/chad/mlx_qsdpa.py:701-702 and 761-764. out is (rows, D) in `dtype` (the scale dtype).
 * round_mode 0: scale*code+bias evaluated exactly and rounded once to dtype;
 * round_mode 1: rounded to dtype after the multiply and again after the add.
 */
int qkv_dequantize(const void* w, const void* scales, const void* biases, void* out,
                   long long rows, int D, int bits, int group_size, int dtype,
                   int round_mode, void* stream);

/*
 * Bytes of scratch that qkv_attention needs for these sizes (n_max = largest key count).
 * The in-kernel merge reads a zero word of the workspace as "not yet written": zero the
 * whole workspace once before the first call (cudaMemset); every call leaves it zero again.
 * After a call reports a device error (QKV_EDEVICE), zero it again. One workspace serves
 * one stream at a time.
 */
size_t qkv_workspace_size(int B, int HQ, int HKV, int S, int D, int n_max, int bits,
                          int group_size);

/*
 * Attention of S query tokens per head over the quantized cache; replaces the
 * reference's qsdpa(q, k_quant, v_quant, scale, n) (src/chad/mlx_qsdpa.py:572-630) and
 * its S>1 dequantize + fused-SDPA branch (src/chad/mlx_qsdpa.py:751-766).
 *
 *   q:        (B, HQ, S, D) in dtype, contiguous; HQ % HKV == 0 (GQA head h uses kv
 *             head h / (HQ/HKV))
 *   kw..vb:   the cache tuples described at the top of this file
 *   out:      see out_kind
 *   n, lens:  keys held here: lens[b] (device int32[B]) when lens != NULL, else n for all b
 *   pos_base: device int32[B] absolute position of this buffer's key 0 (NULL = 0); lets a
 *             sequence shard on one GPU apply the causal rule of the whole sequence
 *   total_lens: device int32[B] full sequence length for the causal rule (NULL = lens/n)
 *   scale:    softmax scale applied to q.k
 *   mask:     QKV_MASK_* ; for BOOL / ADDITIVE, element (b,h,s,k) is read at
 *             mask + b*mask_sb + h*mask_sh + s*mask_sq + k, for k < mask_nk (mask_nk >= key
 *             count); a stride of 0 broadcasts
 *   splits:   split count along the keys (0 = choose from the SM count)
 *   workspace: >= qkv_workspace_size(B, HQ, HKV, S, D, max key count, bits, group_size),
 *             all zero before the first call (every call leaves it zero)
 */
int qkv_attention(const void* q, const void* kw, const void* ks, const void* kb,
                  const void* vw, const void* vs, const void* vb, void* out,
                  int B, int HQ, int HKV, int S, int D, int NP, int n, const int* lens,
                  const int* pos_base, const int* total_lens, int bits, int group_size,
                  int dtype, float scale, int mask_kind, const void* mask, int mask_nk,
                  long long mask_sb, long long mask_sh, long long mask_sq, int out_kind,
                  int splits, void* workspace, size_t ws_bytes, void* stream);

/*
 * Pass 1 only: write the per-split partial rows of qkv_attention without merging them
 * (the reference's pass-1 contract, src/chad/mlx_qsdpa.py:73-209: per block of keys the
 * (max, sum, un-normalised output) of every query row). parts receives
 * [*n_parts][B*HQ*S][D+4] floats, rows laid out as in QKV_OUT_PARTIAL; parts_bytes must be
 * >= qkv_workspace_size(...) for these sizes. *n_parts (host int) receives the split count.
 * Arguments otherwise as in qkv_attention. Merge with qkv_combine.
 */
int qkv_partials(const void* q, const void* kw, const void* ks, const void* kb,
                 const void* vw, const void* vs, const void* vb, float* parts,
                 size_t parts_bytes, int* n_parts, int B, int HQ, int HKV, int S, int D,
                 int NP, int n, const int* lens, const int* pos_base, const int* total_lens,
                 int bits, int group_size, int dtype, float scale, int mask_kind,
                 const void* mask, int mask_nk, long long mask_sb, long long mask_sh,
                 long long mask_sq, int splits, void* stream);

/*
 * Merge n_parts partial results (QKV_OUT_PARTIAL rows) per query row: the pass-2
 * log-sum-exp combine of src/chad/mlx_qsdpa.py:233-258, used to merge sequence shards
 * gathered from several GPUs. parts: float [n_parts][rows][D+4]; out: (rows, D) in
 * out_dtype when out_kind == QKV_OUT_NORMALIZED, else one merged partial row each.
 */
int qkv_combine(const float* parts, int n_parts, long long rows, int D, void* out,
                int out_dtype, int out_kind, void* stream);

/*
 * Cross-GPU merge of sequence shards over peer memory, one kernel per rank: the rank's
 * partial rows (`parts`, rows x (D+4) floats, QKV_OUT_PARTIAL layout, e.g. qkv_attention's
 * output over its key shard) are written straight into every rank's receive buffer over
 * NVLink, each float paired with the call's flag in one 64-bit word; the kernel then reads
 * every rank's rows of this call as they land (bounded wait) and merges them with the pass-2
 * rule of src/chad/mlx_qsdpa.py:233-258 into `out` (QKV_OUT_NORMALIZED: rows x D in
 * out_dtype; QKV_OUT_PARTIAL: one merged partial row each). Replaces an all_gather
 * collective plus qkv_combine; every rank calls it in the same order with the same rows.
 *   peer_bufs: device array of `world` pointers, rank p's receive buffer as mapped in this
 *              process (e.g. by CUDA IPC); my_buf = peer_bufs[rank]
 *   buffers:   qkv_gather_buffer_size(rows, D, world) bytes each, zero before the first
 *              call; their call counters only grow, so no host-side epoch is needed. After
 *              a wait gave up (qkv_device_status), zero every rank's buffer again with every
 *              rank idle before relying on the merge.
 */
size_t qkv_gather_buffer_size(long long rows, int D, int world);
/* Receive buffers for qkv_gather_combine: qkv_peer_alloc makes a zeroed device buffer on
 * the current device and, when ipc_handle is non-null, writes its QKV_IPC_HANDLE_BYTES
 * CUDA IPC handle there for the other ranks; qkv_peer_open maps a peer's buffer from its
 * handle; qkv_peer_free releases either (opened = 1 for a mapping). Free the own buffer
 * only after every peer has closed its mapping of it. */
#define QKV_IPC_HANDLE_BYTES 64
int qkv_peer_alloc(size_t bytes, void** ptr, void* ipc_handle);
int qkv_peer_open(const void* ipc_handle, void** ptr);
int qkv_peer_free(void* ptr, int opened);
int qkv_gather_combine(const float* parts, long long rows, int D, void* const* peer_bufs,
                       void* my_buf, int world, int rank, void* out, int out_dtype,
                       int out_kind, void* stream);

/*
 * Prefill over the prefix cache: quantize-append the S new tokens' K/V at [offset,
 * offset+S) (the cache quantizes before attention runs, src/chad/engine.py:941-990), then
 * attend the S queries over all offset+S keys, causal within the new chunk.
 * k_new / v_new: (B, HKV, S, D) in dtype. Other arguments as in qkv_attention.
 * A decode step (one query-row group per kv head) is a single kernel launch: the attention
 * kernel writes the new rows into the cache itself, bit-identical to qkv_quantize_append.
 */
int qkv_prefill(const void* q, const void* k_new, const void* v_new, void* kw, void* ks,
                void* kb, void* vw, void* vs, void* vb, void* out, int B, int HQ, int HKV,
                int S, int D, int NP, int offset, int bits, int group_size, int dtype,
                float scale, void* workspace, size_t ws_bytes, void* stream);

/*
 * qkv_attention without a workspace argument, for callers that cannot allocate device
 * memory (an FFI host with no CUDA allocator of its own, or an engine whose HBM is reserved
 * up front by a fixed-budget pool). No counterpart in the reference: the reference's
 * kernels allocate their outputs through MLX.
 *
 * The split partials live in a 4 MiB static scratch array inside libqkv.so (held on every
 * GPU that loads the library, until exit); calls whose partials need more return
 * QKV_EWORKSPACE with a message naming both sizes. The first call on a device looks up the
 * array's address (cudaGetSymbolAddress) and should come before any stream capture. All
 * calls on a device share the array: calls that overlap on the GPU race, so serialize them.
 * After qkv_device_status reports QKV_EDEVICE, call qkv_device_status(stream, 1): it zeroes
 * the array again. Arguments and results are those of qkv_attention.
 */
int qkv_attention_noalloc(const void* q, const void* kw, const void* ks, const void* kb,
                          const void* vw, const void* vs, const void* vb, void* out, int B,
                          int HQ, int HKV, int S, int D, int NP, int n, const int* lens,
                          const int* pos_base, const int* total_lens, int bits,
                          int group_size, int dtype, float scale, int mask_kind,
                          const void* mask, int mask_nk, long long mask_sb, long long mask_sh,
                          long long mask_sq, int out_kind, int splits, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CHAD_B200_QKV_H */
