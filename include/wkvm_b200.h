/*
 * wkvm_b200 — C ABI of the B200 (sm_100a) state-slot hot path of wkvm.
 *
 * The path: the RWKV-7 WKV recurrence (a diagonal-plus-low-rank "DPLR" delta
 * rule) and its gated-delta-rule (GDN) sibling, over fixed-size fp32
 * per-request state slots, plus the slot copies around it.
 *
 * Conventions shared by every entry point:
 *   - all tensor pointers are device pointers (snapshot/restore also take a
 *     pinned host pointer, named as such), row-major, contiguous;
 *   - activations are [B, T, H, D] with element type `dtype` (WKVM_DTYPE_*);
 *   - recurrent states are fp32 [.., H, K, V], element h[k][v] (k rows, v
 *     contiguous), the layout of fla and of wkvm's RWKV7StateBank.wkv;
 *   - a "slot bank layer" is the fp32 tensor bank.wkv[layer] of shape
 *     [num_slots, H, K, V] where num_slots counts the reserved padding slot 0
 *     (wkvm allocates S+1 rows for S usable slots);
 *   - slot ids are int32 device arrays; ids must lie in [0, num_slots) and a
 *     batch must not name one slot twice (the host wrapper checks this; the
 *     kernels re-check the range and skip out-of-range rows, reporting
 *     WKVM_ERR_SLOT_RANGE into `status`);
 *   - `status` is an optional device int32 (may be NULL) that receives the
 *     first device-side error; it is never cleared by the library;
 *   - every call is asynchronous on `stream` (a cudaStream_t; NULL = legacy
 *     default stream) and returns 0 or a negative WKVM_ERR_* code for
 *     argument errors found on the host before anything is launched.
 *
 * Reference citations use fla = flash-linear-attention 0.5.1 (the package
 * wkvm's RWKV-7 model delegates its WKV arithmetic to) and wkvm = xiaol/wkvm.
 */
#ifndef WKVM_B200_H_
#define WKVM_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* wkvm_stream_t; /* == cudaStream_t */

enum {
  WKVM_OK = 0,
  WKVM_ERR_INVALID_ARG = -1,  /* null pointer, negative size, bad flag */
  WKVM_ERR_SHAPE = -2,        /* head dim / shape not supported */
  WKVM_ERR_DTYPE = -3,        /* dtype code not supported */
  WKVM_ERR_SLOT_RANGE = -4,   /* slot id outside [0, num_slots) */
  WKVM_ERR_DUPLICATE = -5,    /* one slot named twice in a batch */
  WKVM_ERR_CUDA = -6,         /* a CUDA runtime call failed */
  WKVM_ERR_ALIGN = -7,        /* pointer or row size not 16-byte aligned */
  WKVM_ERR_UNSUPPORTED = -8,  /* option not implemented */
  WKVM_ERR_TIMEOUT = -9,      /* bounded wait ran out */
  WKVM_ERR_SCRATCH = -10      /* request larger than a static scratch array */
};

enum { WKVM_DTYPE_F32 = 0, WKVM_DTYPE_BF16 = 1, WKVM_DTYPE_F16 = 2 };

/* OR-ed into the `dtype` argument of the gated-delta-rule entry points: the
 * per-token gates g and beta are fp32 while q, k, v and o have the dtype in
 * the low byte (fla's GDN layers commonly compute g in fp32; fla's kernels
 * load every pointer in its own dtype). The 16-bit chunk paths then stay on
 * the tensor cores. */
#define WKVM_GATES_F32 0x100

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int wkvm_version(void);

/* Static text for a WKVM_ERR_* code. */
const char* wkvm_strerror(int code);

/* ------------------------------------------------------------------------
 * RWKV-7 recurrent form (decode, and short prefill tails).
 *
 * Replaces fla `fused_mul_recurrent_rwkv7` (fla/ops/rwkv7/fused_recurrent.py:240,
 * kernel :34-129, decode branch :88-102), called by fla's RWKV7Attention at
 * fla/layers/rwkv7.py:323-334 with scale=1. Per token, per head:
 *   sa[v] = sum_k (-kk[k]) h[k][v]            (pre-update state)
 *   h[k][v] = exp(w[k]) h[k][v] + kk[k] a[k] sa[v] + k[k] v[v]
 *   o[v]   = sum_k r[k] scale h[k][v]          (post-update state)
 * w is the log-decay. `h0` (optional, [N,H,K,V]) is the initial state, `ht`
 * (optional) receives the final state; h0 == ht is allowed (in-place).
 * cu_seqlens (optional, int64 device [N+1]) selects varlen mode with B == 1.
 * ------------------------------------------------------------------------ */
int wkvm_fused_mul_recurrent_rwkv7(
    const void* r, const void* w, const void* k, const void* v,
    const void* kk, const void* a, void* o,
    const float* h0, float* ht, const int64_t* cu_seqlens,
    int32_t B, int32_t T, int32_t H, int32_t K, int32_t V,
    float scale, int32_t dtype, int32_t* status, wkvm_stream_t stream);

/* General DPLR recurrent form: replaces fla `fused_recurrent_rwkv7` /
 * `fused_recurrent_dplr_delta_rule` (fla/ops/rwkv7/fused_recurrent.py:183,
 * fla/ops/generalized_delta_rule/dplr/fused_recurrent.py) with explicit a, b:
 *   h = exp(w) h + b (a^T h) + k v^T ;  o = h^T (r scale)                  */
int wkvm_fused_recurrent_dplr(
    const void* r, const void* w, const void* k, const void* v,
    const void* a, const void* b, void* o,
    const float* h0, float* ht, const int64_t* cu_seqlens,
    int32_t B, int32_t T, int32_t H, int32_t K, int32_t V,
    float scale, int32_t dtype, int32_t* status, wkvm_stream_t stream);

/* Slot-native RWKV-7 decode: same arithmetic as
 * wkvm_fused_mul_recurrent_rwkv7 (scale 1), but the state of batch row i is
 * read from and written back to bank_layer[slot_ids[i]] in place. Replaces the
 * gather -> fla kernel -> scatter sequence of wkvm RWKV7StateBank.gather_cache
 * (wkvm/runner/state.py:63-83), fla fused_mul_recurrent_rwkv7 and
 * RWKV7StateBank.scatter_cache (wkvm/runner/state.py:85-97) for one layer.
 * T >= 1 tokens per row are applied in order (T > 1: fla's T-loop branch,
 * fused_recurrent.py:103-125). Inputs [B,T,H,K]; o [B,T,H,V].             */
int wkvm_wkv7_decode_slots(
    const void* r, const void* w, const void* k, const void* v,
    const void* kk, const void* a, void* o,
    float* bank_layer, int64_t num_slots, const int32_t* slot_ids,
    int32_t B, int32_t T, int32_t H, int32_t K, int32_t V,
    int32_t dtype, int32_t* status, wkvm_stream_t stream);

/* Opt-in (process-wide, off by default) overlap of consecutive
 * wkvm_wkv7_decode_slots and wkvm_wkv7_timemix_decode_slots launches with
 * programmatic dependent launch: a launch's CTAs may start while the
 * previous kernel in the stream drains, read their slot ids and state, and
 * only then wait for it before reading their inputs. A launch lets the
 * next one start only after its own wait has returned, so a launch never
 * runs beside any kernel older than its immediate predecessor. Contract while
 * enabled: the kernel launched immediately before such a call on the same
 * stream does not write that call's slot ids or those slots' rows of that
 * layer (true for a loop over layers, where each launch touches another
 * layer, and for a projection GEMM ahead of the time-mix core). Returns the
 * previous setting. No counterpart in the reference. */
int wkvm_set_decode_overlap(int32_t enable);

/* Token-shift + lerp prologue of RWKV-7 single-token decode, with the
 * token-shift state read and written in place by slot id. For row b
 * (slot s = slot_ids[b]) and channel d: delta = shift[s][d] - x[b][d]
 * (rounded to the input dtype, as fla's token_shift stores it),
 * out[i][b][d] = x[b][d] + delta * mixes[i][d] for i < n_mix (n_mix <= 6),
 * then shift[s][d] = x[b][d]. x is [B, D], out [n_mix, B, D], each mix [D],
 * slot rows slot_stride bytes apart (bank.shift[layer, family] rows).
 * Replaces fla token_shift with a cache (fla/modules/token_shift.py:521) +
 * torch_addcmul_rwkv7 (fla/ops/rwkv7/fused_addcmul.py:290) in RWKV7Attention,
 * the same pair with x_k in RWKV7FeedForward
 * (fla/models/rwkv7/modeling_rwkv7.py:98-115), and wkvm's gather/scatter of
 * the shift family (wkvm/runner/state.py:63-97). bf16/fp16, D % 8 == 0. */
int wkvm_wkv7_shift_mix_slots(
    const void* x, void* out, void* shift_rows, int64_t slot_stride,
    int64_t num_slots, const int32_t* slot_ids, const void* const* mixes,
    int32_t n_mix, int32_t B, int32_t D, int32_t dtype,
    int32_t* status, wkvm_stream_t stream);

/* Fused RWKV-7 time-mix decode core: the whole of fla RWKV7Attention between
 * its projections and o_proj for one token, around an in-place slot update
 * (fla/layers/rwkv7.py:270-349): w = -0.6065306597126334 sigmoid(w_raw),
 * a = sigmoid(a_raw), v = lerp(v, v_first, sigmoid(v_raw)) (v_first and
 * v_raw NULL for layer 0), kk = l2norm(k k_k) per head, k' = k + k (a-1) k_a,
 * the WKV step on bank_layer[slot_ids[i]], then GroupNorm per head
 * (gn_w, gn_b, gn_eps), o += (sum r k' r_k) v, o *= g. Activations are
 * [B, H*64] rows; k_k, k_a, r_k, gn_w, gn_b are [H*64] parameters in the
 * same dtype. Head dim 64. */
int wkvm_wkv7_timemix_decode_slots(
    const void* r, const void* w_raw, const void* k, const void* v,
    const void* v_first, const void* v_raw, const void* a_raw, const void* g,
    const void* k_k, const void* k_a, const void* r_k, const void* gn_w,
    const void* gn_b, void* o, float* bank_layer, int64_t num_slots,
    const int32_t* slot_ids, int32_t B, int32_t H, int32_t K, float gn_eps,
    int32_t dtype, int32_t* status, wkvm_stream_t stream);

/* ------------------------------------------------------------------------
 * Gated delta rule (GDN) recurrent form.
 *
 * Replaces fla `fused_recurrent_gated_delta_rule`
 * (fla/ops/gated_delta_rule/fused_recurrent.py:291, kernel :28-170) for
 * head-wise g and beta, standard [K,V] state layout:
 *   h = exp(g) h ; v' = beta (v - h^T k) ; h += k v'^T ; o = h^T (q scale)
 * q, k: [B,T,H,K]; v, o: [B,T,HV,V]; g, beta: [B,T,HV]; HV % H == 0 (grouped
 * value heads). use_qk_l2norm != 0 normalises q and k per head in-kernel as
 * fla does (x / sqrt(sum x^2 + 1e-6)).                                    */
int wkvm_fused_recurrent_gated_delta_rule(
    const void* q, const void* k, const void* v, const void* g,
    const void* beta, void* o,
    const float* h0, float* ht, const int64_t* cu_seqlens,
    int32_t B, int32_t T, int32_t H, int32_t HV, int32_t K, int32_t V,
    float scale, int32_t use_qk_l2norm, int32_t dtype,
    int32_t* status, wkvm_stream_t stream);

/* Slot-native GDN decode: state of row i lives at bank_layer[slot_ids[i]]
 * ([num_slots, HV, K, V] fp32) and is updated in place.                   */
int wkvm_gdn_decode_slots(
    const void* q, const void* k, const void* v, const void* g,
    const void* beta, void* o,
    float* bank_layer, int64_t num_slots, const int32_t* slot_ids,
    int32_t B, int32_t T, int32_t H, int32_t HV, int32_t K, int32_t V,
    float scale, int32_t use_qk_l2norm, int32_t dtype,
    int32_t* status, wkvm_stream_t stream);

/* ------------------------------------------------------------------------
 * Chunked prefill (WY / UT-transform form, 64-token chunks, tcgen05 tf32
 * tensor cores, fp32 accumulation). Same arithmetic as the recurrent forms
 * above, reassociated by chunk.
 *
 * Replaces fla `chunk_rwkv7` (fla/ops/rwkv7/chunk.py:13) ->
 * `chunk_dplr_delta_rule` (fla/ops/generalized_delta_rule/dplr/chunk.py:442,
 * forward :33-135), called by fla's RWKV7Attention for seq_len >= 64
 * (fla/layers/rwkv7.py:305-321) with a = -kk, b = kk * a_gate, scale 1.
 * K == V == 64 runs the tensor-core kernel; other head sizes run the
 * recurrent kernel. The chunk kernel requires |sum of w| over any 32
 * consecutive tokens <= 80 (RWKV-7's w = -0.6065 sigmoid(.) keeps it under
 * 20) and reports WKVM_ERR_UNSUPPORTED in `status` otherwise.
 * ------------------------------------------------------------------------ */
int wkvm_chunk_dplr(
    const void* r, const void* w, const void* k, const void* v,
    const void* a, const void* b, void* o,
    const float* h0, float* ht, const int64_t* cu_seqlens,
    int32_t B, int32_t T, int32_t H, int32_t K, int32_t V,
    float scale, int32_t dtype, int32_t* status, wkvm_stream_t stream);

/* Slot-native RWKV-7 prefill: the initial state of sequence i is read from
 * bank_layer[slot_ids[i]] and the final state written back there. Replaces
 * wkvm RWKV7Runner.prefill's gather -> chunk_rwkv7 -> scatter round trip
 * per host chunk (wkvm/runner/runner.py:52-62). Inputs (r, w, k, v, kk,
 * a_gate) as for wkvm_wkv7_decode_slots; cu_seqlens (optional) packs
 * variable-length sequences with B = number of sequences.                 */
int wkvm_wkv7_prefill_slots(
    const void* r, const void* w, const void* k, const void* v,
    const void* kk, const void* a, void* o,
    float* bank_layer, int64_t num_slots, const int32_t* slot_ids,
    const int64_t* cu_seqlens,
    int32_t B, int32_t T, int32_t H, int32_t K, int32_t V,
    int32_t dtype, int32_t* status, wkvm_stream_t stream);

/* Slot-native prefill in fla's general DPLR form (explicit a, b and scale),
 * the arguments fla's RWKV7Attention passes to chunk_rwkv7
 * (fla/layers/rwkv7.py:308-321). Head dim 64 with 16-bit inputs only
 * (WKVM_ERR_UNSUPPORTED otherwise). */
int wkvm_dplr_prefill_slots(
    const void* r, const void* w, const void* k, const void* v,
    const void* a, const void* b, void* o,
    float* bank_layer, int64_t num_slots, const int32_t* slot_ids,
    const int64_t* cu_seqlens,
    int32_t B, int32_t T, int32_t H, int32_t K, int32_t V,
    float scale, int32_t dtype, int32_t* status, wkvm_stream_t stream);

/* Chunked GDN prefill: replaces fla `chunk_gated_delta_rule`
 * (fla/ops/gated_delta_rule/chunk.py:365, forward :29-116) for head-wise g
 * and beta, [K,V] state layout. Arguments as for
 * wkvm_fused_recurrent_gated_delta_rule, plus a device workspace the caller
 * owns. K == V == 128 with 16-bit inputs runs on the tcgen05 tensor core:
 * with a workspace of at least one window (see
 * wkvm_gdn_chunk_workspace_bytes) as two launches, a chunk-parallel WY
 * kernel and a sequential state pass; without one as a single kernel (one
 * CTA per sequence, value head and half of V). Other shapes run the
 * recurrent kernel. The workspace is 256-byte aligned or ignored. The
 * two-launch path keeps its per-chunk records in fp16 (the tf32
 * significand) and multiplies in kind::f16; a record value beyond fp16's
 * range (|v| above ~6e4) is reported as WKVM_ERR_UNSUPPORTED in `status`,
 * and such inputs run without a workspace (tf32 operands throughout). */
int wkvm_chunk_gated_delta_rule(
    const void* q, const void* k, const void* v, const void* g,
    const void* beta, void* o,
    const float* h0, float* ht, const int64_t* cu_seqlens,
    int32_t B, int32_t T, int32_t H, int32_t HV, int32_t K, int32_t V,
    float scale, int32_t use_qk_l2norm, int32_t dtype,
    void* workspace, int64_t workspace_bytes,
    int32_t* status, wkvm_stream_t stream);

/* Workspace bytes for the two-launch GDN prefill of nseq sequences of at
 * most T tokens (T = total tokens with cu_seqlens) in one window; 0 when the
 * shape does not take that path. A smaller workspace (at least
 * nseq*HV*(64 KiB + one chunk record) bytes) processes the chunks in
 * windows. */
int64_t wkvm_gdn_chunk_workspace_bytes(int32_t nseq, int32_t T, int32_t HV, int32_t K, int32_t V);

/* wkvm_chunk_gated_delta_rule for callers that cannot allocate device
 * memory (a host whose device memory belongs to its own pool, or a cgo / JNI
 * embedding with no allocator, where cudaMalloc would also synchronise the
 * device mid-serving). No counterpart exists in the reference: it is the
 * two-launch path with its workspace in a 64 MiB array that the library
 * keeps on every GPU that loads it, until the process exits. Arguments as
 * for wkvm_chunk_gated_delta_rule without the workspace; K == V == 128 and
 * 16-bit inputs only (WKVM_ERR_SHAPE / WKVM_ERR_DTYPE otherwise). Longer
 * inputs run in windows of chunks; WKVM_ERR_SCRATCH when even one window
 * does not fit (about nseq * HV > 480). Runs on the current device; the
 * first call on each device, and the first after a cudaDeviceReset, looks
 * up the array's device address (cudaGetSymbolAddress), so make that first
 * call before any stream capture. All calls share the array: calls that overlap on the GPU (other
 * streams, other host threads) race; sequential calls need nothing cleared
 * between them, since each call writes every byte it reads. */
int wkvm_chunk_gated_delta_rule_static(
    const void* q, const void* k, const void* v, const void* g,
    const void* beta, void* o,
    const float* h0, float* ht, const int64_t* cu_seqlens,
    int32_t B, int32_t T, int32_t H, int32_t HV, int32_t K, int32_t V,
    float scale, int32_t use_qk_l2norm, int32_t dtype,
    int32_t* status, wkvm_stream_t stream);

/* Slot-native chunked GDN prefill: initial and final state of sequence i
 * in bank_layer[slot_ids[i]] ([num_slots, HV, K, V] fp32). No wkvm caller
 * exists (wkvm runs RWKV-7 only); the operator contract is fla's. */
int wkvm_gdn_prefill_slots(
    const void* q, const void* k, const void* v, const void* g,
    const void* beta, void* o,
    float* bank_layer, int64_t num_slots, const int32_t* slot_ids,
    const int64_t* cu_seqlens,
    int32_t B, int32_t T, int32_t H, int32_t HV, int32_t K, int32_t V,
    float scale, int32_t use_qk_l2norm, int32_t dtype,
    void* workspace, int64_t workspace_bytes,
    int32_t* status, wkvm_stream_t stream);

/* ------------------------------------------------------------------------
 * Slot copies. A state family tensor is viewed as [outer, num_slots, row]:
 * bank.wkv [L, S+1, H*K*V fp32] has outer = L; bank.shift [L, 2, S+1, D]
 * has outer = 2L. `outer_stride` and `slot_stride` are in bytes, `row_bytes`
 * is the bytes of one slot's row within one outer index. Copies are bitwise.
 * Row bytes, strides and base pointers must be 16-byte aligned.
 * ------------------------------------------------------------------------ */

/* Fork: rows of dst_ids[i] <- rows of src_ids[i] (all outer indices).
 * Defines on device what wkvm StateArena.fork leaves to the runner
 * (wkvm/core/arena.py:82-92). src and dst sets must not overlap. */
int wkvm_slot_copy(void* base, int64_t outer, int64_t outer_stride,
                   int64_t slot_stride, int64_t row_bytes, int64_t num_slots,
                   const int32_t* src_ids, const int32_t* dst_ids, int32_t n,
                   int32_t* status, wkvm_stream_t stream);

/* Zero the rows of ids[i]: wkvm RWKV7StateBank.zero_slots
 * (wkvm/runner/state.py:50-54). */
int wkvm_slot_zero(void* base, int64_t outer, int64_t outer_stride,
                   int64_t slot_stride, int64_t row_bytes, int64_t num_slots,
                   const int32_t* ids, int32_t n,
                   int32_t* status, wkvm_stream_t stream);

/* Snapshot: packed[i][o][:] <- base[o][ids[i]][:] for n slots into a packed
 * buffer [n, outer, row_bytes] that may be pinned, device-mapped host memory
 * (the layout of wkvm StateStore.save's bank.wkv[:, slot] host copy,
 * wkvm/store.py:130-131,248-252). */
int wkvm_slot_snapshot(const void* base, int64_t outer, int64_t outer_stride,
                       int64_t slot_stride, int64_t row_bytes,
                       int64_t num_slots, const int32_t* ids, int32_t n,
                       void* packed, int32_t* status, wkvm_stream_t stream);

/* Restore: base[o][ids[i]][:] <- packed[i][o][:] (wkvm StateStore.load,
 * wkvm/store.py:151-153). */
int wkvm_slot_restore(void* base, int64_t outer, int64_t outer_stride,
                      int64_t slot_stride, int64_t row_bytes,
                      int64_t num_slots, const int32_t* ids, int32_t n,
                      const void* packed, int32_t* status,
                      wkvm_stream_t stream);

/* Gather / scatter with an explicit layout of the packed side: element
 * (outer o, batch index i) of the packed buffer starts at
 * o * dst_outer_stride + i * dst_index_stride bytes (snapshot/restore are the
 * case dst_index_stride = outer * row_bytes). Used to hand a model one
 * contiguous [n, row] view per layer of a family (the reference gathers with
 * one index_select per layer and family, wkvm/runner/state.py:76-79). */
int wkvm_slot_gather(const void* base, int64_t outer, int64_t outer_stride,
                     int64_t slot_stride, int64_t row_bytes, int64_t num_slots,
                     const int32_t* ids, int32_t n, void* dst, int64_t dst_outer_stride,
                     int64_t dst_index_stride, int32_t* status, wkvm_stream_t stream);
int wkvm_slot_scatter(void* base, int64_t outer, int64_t outer_stride,
                      int64_t slot_stride, int64_t row_bytes, int64_t num_slots,
                      const int32_t* ids, int32_t n, const void* src, int64_t src_outer_stride,
                      int64_t src_index_stride, int32_t* status, wkvm_stream_t stream);

/* Live migration: rows of dst_ids[i] in dst_base (a peer GPU's bank, peer
 * access enabled by the caller) <- rows of src_ids[i] in src_base. Both
 * banks share outer/strides/row size. Plain peer stores over NVLink; launch
 * on the source GPU's stream. No counterpart in the reference, whose README
 * only plans it. */
int wkvm_slot_migrate(const void* src_base, void* dst_base, int64_t outer,
                      int64_t outer_stride, int64_t slot_stride,
                      int64_t row_bytes, int64_t src_num_slots,
                      int64_t dst_num_slots, const int32_t* src_ids,
                      const int32_t* dst_ids, int32_t n, int32_t* status,
                      wkvm_stream_t stream);

/* Self-test of the tensor-core layer the prefill kernels use: one tile
 * D[128,N] = A[128,64] B[N,64]^T with tcgen05.mma kind::tf32, fp32 row-major
 * device buffers, N in {64, 128}; a_in_tmem != 0 feeds A from tensor
 * memory instead of shared memory. No counterpart in the reference. */
int wkvm_selftest_tf32_mma(const float* A, const float* B, float* D, int32_t N,
                           int32_t a_in_tmem, int32_t* status, wkvm_stream_t stream);

/* State mutation rules on device: for each i, rows of dst_ids[i] <-
 * c1 * rows(a_ids[i]) + c2 * rows(b_ids[i]) (b_ids NULL: c1 * rows(a_ids[i])),
 * computed in fp32 with separately rounded products and sum, then rounded to
 * the family's dtype (dtype = WKVM_DTYPE_*). Bitwise equal to wkvm's
 * StateStore rules applied with torch: merge (wkvm/store.py:260-268,
 * c1 = 1 - weight, c2 = weight) and decay (wkvm/store.py:298-305,
 * c1 = alpha, wkv family only). dst may equal a (in place); a slot may not be
 * both a destination and a source of another pair in one call. */
int wkvm_slot_affine(void* base, int64_t outer, int64_t outer_stride,
                     int64_t slot_stride, int64_t row_bytes, int64_t num_slots,
                     const int32_t* dst_ids, const int32_t* a_ids, const int32_t* b_ids,
                     int32_t n, float c1, float c2, int32_t dtype, int32_t* status,
                     wkvm_stream_t stream);

/* Enables `device` -> `peer` access (cudaDeviceEnablePeerAccess with
 * `device` current); already-enabled counts as success. Needed once per pair
 * before wkvm_slot_migrate writes into the peer's bank. */
int wkvm_enable_peer_access(int32_t device, int32_t peer);

#ifdef __cplusplus
}
#endif

#endif /* WKVM_B200_H_ */
