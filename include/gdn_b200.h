/*
 * gdn_b200.h — C ABI of the B200 (sm_100a) Gated DeltaNet hot path.
 *
 * Plain pointers and sizes; no framework types.  Every buffer is device
 * memory owned by the caller (destination-passing style, outputs last), and
 * no entry point allocates device memory or synchronises the stream: each
 * call validates its arguments on the host, enqueues its kernel on `stream`
 * (a cudaStream_t; NULL = the legacy default stream) and returns.
 *
 * Layouts (all contiguous, row-major, D = head_dim = 128):
 *   decode : q, k [B,1,H_qk,D] bf16;  v [B,1,H_v,D] bf16;  a, b [B,1,H_v] bf16;
 *            state, new_state [B,H_v,D(v),D(k)] fp32 (k-last);  output [B,1,H_v,D] bf16.
 *   prefill: q, k [T,H_qk,D] bf16;  v [T,H_v,D] bf16;  a, b [T,H_v] bf16 (packed tokens);
 *            cu_seqlens [N+1] int32 or int64;  state, new_state [N,H_v,D,D] fp32;
 *            output [T,H_v,D] bf16.
 *   A_log, dt_bias: [H_v] fp32.   H_v % H_qk == 0 (v-head h reads qk-head h / (H_v/H_qk)).
 *
 * Semantics (identical to the reference's TVM-FFI `kernel` entry points):
 *   scale == 0      -> 1/sqrt(D)                               (ref solution/cuda/kernel.cu:115-118)
 *   state == NULL   -> zero initial state                      (ref kernel.cu:135-139)
 *   new_state may alias state (in-place update); output must not alias any input.
 *   prefill: an empty sequence copies its initial state        (ref kernel_prefill.cu:61-66)
 *
 * Return value: GDN_B200_OK, or an error code whose message is available from
 * gdn_b200_last_error() on the calling thread.
 */
#ifndef GDN_B200_H_
#define GDN_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GDN_B200_OK 0
#define GDN_B200_ERR_INVALID_ARGUMENT 1  /* shape, pointer, alignment or head-layout error */
#define GDN_B200_ERR_CUDA 2              /* a CUDA runtime/driver call failed */

/* Device status bits (read with gdn_b200_device_status). */
#define GDN_B200_STATUS_TMA_TIMEOUT 1u   /* a prefill TMA wait exceeded its bound */
#define GDN_B200_STATUS_MMA_TIMEOUT 2u   /* a prefill tensor-core wait exceeded its bound */
#define GDN_B200_STATUS_BAD_SEQLENS 4u   /* cu_seqlens not non-decreasing within [0, total_tokens] */
#define GDN_B200_STATUS_BAD_INDEX 8u     /* a state-pool index was >= pool_size */
#define GDN_B200_STATUS_SELFTEST_WAIT 16u /* gdn_b200_selftest_wait_timeout's wait ran out */

/*
 * One T=1 decode step for `batch` sequences.
 * Replaces the reference's TVM-FFI `kernel` of solution/cuda/kernel.cu:101-150
 * (GDNDecodeKernel(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state)),
 * with the tensor extents passed explicitly.
 */
int gdn_b200_decode(const void* q, const void* k, const void* v, const float* state,
                    const float* A_log, const void* a, const float* dt_bias, const void* b,
                    double scale, void* output, float* new_state,
                    int64_t batch, int32_t num_qk_heads, int32_t num_v_heads, int32_t head_dim,
                    void* stream);

/*
 * Decode of `seq_len` >= 1 tokens per sequence against a state pool: the
 * serving-side forms of the step above.  No counterpart in the reference's
 * contest kit; the semantics are those of the next definitions of the same
 * family: FlashInfer's pooled decode
 * (gated_delta_rule_decode_pretranspose with initial_state, initial_state_indices,
 * output_state_indices; site flashinfer/gdn_decode.py:117-200) and the MTP /
 * speculative-verify definition (site flashinfer/trace/templates/gdn.py:378-466).
 *
 *   q, k [B,T,H_qk,D] bf16;  v [B,T,H_v,D] bf16;  a, b [B,T,H_v] bf16;
 *   output [B,T,H_v,D] bf16;
 *   state_pool, new_state_pool [P,H_v,D(v),D(k)], fp32 (state_is_bf16 = 0) or bf16 (= 1);
 *     new_state_pool may alias state_pool (in-place, the serving case); only the slots
 *     named by the indices are written;
 *   read_indices, write_indices [B] int32 (indices_are_int64 = 0) or int64 (= 1):
 *     entry b reads slot read_indices[b] and writes its final state to slot
 *     write_indices[b] (write_indices = NULL: the read slot);
 *   intermediate_states: NULL, or [P,T,H_v,D,D] of the state type; the state after
 *     token t of entry b is stored at [read_indices[b], t] (for rollback).
 * A negative index marks a padding entry: its outputs are zero and no state is read or
 * written.  An index >= pool_size is treated as padding and sets
 * GDN_B200_STATUS_BAD_INDEX.  Entries must not share a write slot, and no entry may
 * write a slot another entry reads.  The recurrence runs in fp32; a bf16 pool is
 * rounded once per stored state.
 */
int gdn_b200_decode_pool(const void* q, const void* k, const void* v,
                         const void* state_pool, void* new_state_pool, int32_t state_is_bf16,
                         const void* read_indices, const void* write_indices,
                         int32_t indices_are_int64, void* intermediate_states,
                         const float* A_log, const void* a, const float* dt_bias, const void* b,
                         double scale, void* output, int64_t batch, int64_t seq_len,
                         int64_t pool_size, int32_t num_qk_heads, int32_t num_v_heads,
                         int32_t head_dim, void* stream);

/* Capacity (bytes) of the record ring that gdn_b200_prefill works in: 1 GiB,
 * the records of about 42,000 tokens of one sequence at qk16_v32 (0.6 % of a
 * B200's HBM).  (The host side of a device array of 2 GiB or more does not
 * link with the default small code model.) */
#define GDN_B200_PREFILL_RING_BYTES (1024ull << 20)

/*
 * Chunked (C=64) prefill over `num_seqs` packed variable-length sequences.
 * Replaces the reference's TVM-FFI `kernel` of solution/cuda/kernel_prefill.cu:300-339
 * (GDNPrefillKernel(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output,
 * new_state)).  `cu_seqlens` is device memory of int32 (cu_seqlens_is_int64 = 0) or
 * int64 (= 1) entries; `total_tokens` is the packed token extent T of q/k/v/a/b/output.
 *
 * Like the reference kernel it allocates nothing.  It runs the two-stage path
 * of gdn_b200_prefill_ws in a record ring that is part of this library's
 * device image (GDN_B200_PREFILL_RING_BYTES on every GPU that loads the
 * library, held until the process exits): when the problem's records do not
 * all fit, consecutive windows of chunks take turns in the ring.  Results are
 * bit-identical to gdn_b200_prefill_ws.  Calls on one device share the ring;
 * each call's stream waits (on the GPU, through an event) for the previous
 * call's kernels, so calls from several streams or threads are safe, except
 * under CUDA graph capture, where that handoff is skipped and captured calls
 * must not overlap other calls on the device.  A problem whose chunk tables
 * ((ceil(T/64) + N) x 16 bytes) crowd out two rows of records is rejected with
 * GDN_B200_ERR_INVALID_ARGUMENT.
 */
int gdn_b200_prefill(const void* q, const void* k, const void* v, const float* state,
                     const float* A_log, const void* a, const float* dt_bias, const void* b,
                     const void* cu_seqlens, int32_t cu_seqlens_is_int64, double scale,
                     void* output, float* new_state,
                     int64_t num_seqs, int64_t total_tokens, int32_t num_qk_heads,
                     int32_t num_v_heads, int32_t head_dim, void* stream);

/*
 * The same prefill as one kernel: one CTA per (sequence, v-head) walks its
 * chunks and does each chunk's preparation inline before its recurrence, as
 * the reference kernel's structure does (ref solution/cuda/kernel_prefill.cu:36-298,
 * entry point :300-339).  It needs no workspace at all, but puts all the
 * per-chunk work on the sequential chain (several times slower than the
 * two-stage path for long sequences).  Same arguments and semantics as
 * gdn_b200_prefill; results agree with it to the prefill tolerance, not bitwise
 * (the two paths fold the products differently).
 */
int gdn_b200_prefill_fused(const void* q, const void* k, const void* v, const float* state,
                           const float* A_log, const void* a, const float* dt_bias,
                           const void* b, const void* cu_seqlens, int32_t cu_seqlens_is_int64,
                           double scale, void* output, float* new_state, int64_t num_seqs,
                           int64_t total_tokens, int32_t num_qk_heads, int32_t num_v_heads,
                           int32_t head_dim, void* stream);

/*
 * Bytes of device workspace gdn_b200_prefill_ws needs for this problem size
 * (0 when num_seqs <= 0).  The two-stage prefill keeps one 49 KiB record per
 * (64-token chunk, v-head) plus small chunk tables.  No counterpart in the
 * reference, whose single kernel needs no workspace.
 */
uint64_t gdn_b200_prefill_workspace_size(int64_t num_seqs, int64_t total_tokens,
                                         int32_t num_v_heads);

/*
 * Same contract and results as gdn_b200_prefill (replaces the same reference
 * entry point, solution/cuda/kernel_prefill.cu:300-339) with every record of the
 * call resident in a caller workspace, computed in two stages:
 * the S-independent work of every (chunk, v-head) in parallel across the GPU,
 * then the sequential state recurrence per (sequence, v-head, 64-column V
 * slice).  `workspace` is caller-owned device memory of at least
 * gdn_b200_prefill_workspace_size() bytes, 256-byte aligned; its contents are
 * scratch and must not be shared by calls that overlap on the GPU.
 */
int gdn_b200_prefill_ws(const void* q, const void* k, const void* v, const float* state,
                        const float* A_log, const void* a, const float* dt_bias, const void* b,
                        const void* cu_seqlens, int32_t cu_seqlens_is_int64, double scale,
                        void* output, float* new_state,
                        int64_t num_seqs, int64_t total_tokens, int32_t num_qk_heads,
                        int32_t num_v_heads, int32_t head_dim,
                        void* workspace, uint64_t workspace_bytes, void* stream);

/*
 * Affine state combine of the context-parallel prefill, per head:
 *   out[h] = state[h] * transfer[h] + offset[h]     (128 x 128 fp32, row = v)
 * Over a segment of a sequence the chunked recurrence maps every state row the
 * same affine way, S_end = S_0 * M + N (M: the segment's transfer, the final state
 * of a V = 0 run from the identity; N: its offset, the final state of a run from
 * the zero state), so a rank learns its segment's initial state by folding the
 * (M, N) of the segments before it.  state == NULL means a zero state (out =
 * offset).  out may alias offset but not state or transfer.  All [num_heads, 128,
 * 128] fp32.  No counterpart in the reference, which is single-GPU.
 */
int gdn_b200_state_affine(const float* state, const float* transfer, const float* offset,
                          float* out, int64_t num_heads, void* stream);

/*
 * The two stages of gdn_b200_prefill_ws as separate calls, so that one
 * preparation serves several recurrences over the same tokens (the
 * context-parallel prefill runs three: from the zero state, from the identity
 * with zero values, and from the true initial state).  No counterpart in the
 * reference, whose single kernel does both.
 *
 * gdn_b200_prefill_prepare writes the chunk table and the per-(chunk, v-head)
 * records (everything that depends on q, k, a, b, A_log, dt_bias only) into
 * `workspace` (same size and alignment rules as gdn_b200_prefill_ws).
 *
 * gdn_b200_prefill_recur runs the state recurrence over a workspace that a
 * preceding gdn_b200_prefill_prepare with the same num_seqs / total_tokens /
 * heads filled (earlier on the same stream, or ordered before it); it only
 * reads the workspace, so recurrences may run concurrently on other streams.
 * `k` must be the prepared k.  v == NULL means all-zero values; output == NULL
 * skips the outputs; state == NULL means zero initial states.
 */
int gdn_b200_prefill_prepare(const void* q, const void* k, const float* A_log, const void* a,
                             const float* dt_bias, const void* b, const void* cu_seqlens,
                             int32_t cu_seqlens_is_int64, int64_t num_seqs, int64_t total_tokens,
                             int32_t num_qk_heads, int32_t num_v_heads, int32_t head_dim,
                             void* workspace, uint64_t workspace_bytes, void* stream);
int gdn_b200_prefill_recur(const void* k, const void* v, const float* state, double scale,
                           void* output, float* new_state, int64_t num_seqs, int64_t total_tokens,
                           int32_t num_qk_heads, int32_t num_v_heads, int32_t head_dim,
                           const void* workspace, uint64_t workspace_bytes, void* stream);

/* Capacity (bytes) of the scratch array that gdn_b200_prefill_static uses. */
#define GDN_B200_PREFILL_STATIC_SCRATCH_BYTES (64ull << 20)

/*
 * The two-stage prefill (same arguments, semantics and results as
 * gdn_b200_prefill_ws) for callers that cannot allocate device memory: hosts
 * bound to the reference's fixed `kernel` argument list, which has no slot for
 * a workspace; plugin hosts whose framework owns all device memory and forbids
 * raw cudaMalloc; and serving loops that cannot afford an allocation on the hot
 * path.  It allocates nothing: its workspace is a 64 MiB array inside this
 * library's device image, which every GPU that loads the library holds until
 * the process exits.  A problem whose gdn_b200_prefill_workspace_size() exceeds
 * GDN_B200_PREFILL_STATIC_SCRATCH_BYTES is rejected with
 * GDN_B200_ERR_INVALID_ARGUMENT (with qk16_v32 heads the limit is about 1,300
 * (64-token chunk, v-head) pairs, i.e. roughly 2,500 packed tokens).
 * The first call on a device looks up the array's device address (with that
 * device current); make that first call before any stream capture.  All calls
 * on a device share the one array, so calls that overlap on the GPU (other
 * streams, other host threads) race and corrupt each other's results.
 * No counterpart in the reference, whose single kernel needs no workspace.
 */
int gdn_b200_prefill_static(const void* q, const void* k, const void* v, const float* state,
                            const float* A_log, const void* a, const float* dt_bias,
                            const void* b, const void* cu_seqlens, int32_t cu_seqlens_is_int64,
                            double scale, void* output, float* new_state,
                            int64_t num_seqs, int64_t total_tokens, int32_t num_qk_heads,
                            int32_t num_v_heads, int32_t head_dim, void* stream);

/*
 * Reads (and with clear != 0 resets) the status word that the kernels of
 * this library set on `device` when a bounded device-side wait runs out or a
 * cu_seqlens entry is out of range.  Synchronises the device.  No counterpart
 * in the reference, which performs no device-side checks.
 */
int gdn_b200_device_status(int32_t device, uint32_t* status, int32_t clear);

/*
 * Diagnostic of the device-side failure detection: launches one warp that waits
 * on an mbarrier nothing ever arrives on, with the bounded wait the prefill
 * kernels use but a limit of `limit_ns` nanoseconds (at most 1 s).  The wait
 * runs out, the kernel sets GDN_B200_STATUS_SELFTEST_WAIT and returns; the
 * context stays usable.  No counterpart in the reference.
 */
int gdn_b200_selftest_wait_timeout(uint64_t limit_ns, void* stream);

/*
 * Diagnostic of the chain kernel's failure handling: the recurrence of
 * gdn_b200_prefill_recur (same arguments; scale 1/sqrt(D)) over a workspace a
 * gdn_b200_prefill_prepare call filled, with every bounded wait of the chain
 * kernel limited to `limit_ns` nanoseconds (at most 1 s), and with the loads of
 * each sequence's chunks from its third one on withheld.  The first wait on a
 * withheld stage runs out: that CTA raises its abort flag, every one of its
 * roles leaves its loop, waits (bounded) for its copies and tensor-core
 * operations in flight, the CTA frees its TMEM and returns, and the status
 * word gets GDN_B200_STATUS_TMA_TIMEOUT (or _MMA_TIMEOUT).  Outputs and
 * new_state are then incomplete; the context stays usable.  Sequences of at
 * most two chunks (128 tokens) complete normally.  No counterpart in the
 * reference.
 */
int gdn_b200_selftest_prefill_abort(uint64_t limit_ns, const void* k, const void* v,
                                    const float* state, void* output, float* new_state,
                                    int64_t num_seqs, int64_t total_tokens, int32_t num_qk_heads,
                                    int32_t num_v_heads, int32_t head_dim, const void* workspace,
                                    uint64_t workspace_bytes, void* stream);

/*
 * The device this library launches on from the calling thread: the device of
 * the thread's current CUDA context (set by cudaSetDevice in any runtime of the
 * process, e.g. torch.cuda.device), or -1 if none can be read.  Every entry
 * point launches on, and sets up, this device, so a caller whose tensors live
 * on another device makes that device current first.  No counterpart in the
 * reference.
 */
int32_t gdn_b200_current_device(void);

/* Message of the last failing call on this thread ("" if none). */
const char* gdn_b200_last_error(void);

/* Library ABI version (major * 100 + minor). */
int32_t gdn_b200_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif  /* GDN_B200_H_ */
