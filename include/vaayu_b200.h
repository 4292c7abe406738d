/*
 * vaayu_b200.h -- C ABI of the B200 (sm_100a) fused packed-int4 MoE expert path.
 *
 * One shared library, libvaayu_b200.so, exports these entry points.  They replace the Triton
 * kernels and the torch dequant of archish9/Vaayu's packed-expert path; citations are paths
 * inside that project.  Conventions shared by every entry point:
 *
 *   - All tensor arguments are DEVICE pointers of the current CUDA device; sizes are element
 *     counts; strides are in elements.  Nothing here takes ownership of any buffer.
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream).  Every entry point only
 *     ENQUEUES work on it and returns; it never synchronises and never allocates device memory
 *     (scratch comes from the caller's `workspace`).
 *   - The return value is a status: VY_OK (0) or a negative VY_ERR_* code; vy_last_error()
 *     gives the message of the calling thread's last failure.  Unsupported geometry is
 *     VY_ERR_UNSUPPORTED: there is no fallback path behind any entry point.
 *   - dtype codes are the vy_dtype values below.
 */
#ifndef VAAYU_B200_H
#define VAAYU_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VY_ABI_VERSION 4

enum vy_status {
    VY_OK = 0,
    VY_ERR_UNSUPPORTED = -1, /* geometry / dtype the kernels do not take */
    VY_ERR_INVALID = -2,     /* null pointer, negative size, inconsistent shapes */
    VY_ERR_ALIGNMENT = -3,   /* a pointer or stride breaks the 16-byte rule of a vector load */
    VY_ERR_WORKSPACE = -4,   /* workspace smaller than vy_moe_workspace_size() asked for */
    VY_ERR_CUDA = -5,        /* a CUDA runtime error while enqueueing */
    VY_ERR_DEVICE = -6       /* the current device is not an sm_100 part */
};

enum vy_dtype {
    VY_BF16 = 0,
    VY_F16 = 1,
    VY_F32 = 2,
    VY_E4M3 = 3, /* float8_e4m3fn */
    VY_E8M0 = 4, /* float8_e8m0fnu (power-of-two scales) */
    VY_I32 = 5,
    VY_I64 = 6
};

/* The calling thread's last error message ("" after a success). */
const char* vy_last_error(void);
/* VY_ABI_VERSION of the loaded library. */
int vy_abi_version(void);

/* ── int-b packed dequant helpers ───────────────────────────────────────────────────────── */

/*
 * Inverse of compressed-tensors' pack_to_int32 along the last dim: element j of a word at bits
 * [b*j, b*j+b); out = code - 2^(b-1) as int8.  packed [rows, words_per_row], out [rows, cols].
 * Replaces vaayu/moe_patch.py:668-710 `unpack_int32_to_int8` (bits dividing 32).
 */
int vy_unpack_int32_to_int8(const int32_t* packed, int64_t rows, int64_t words_per_row,
                            int32_t bits, int64_t cols, int8_t* out, void* stream);

/*
 * One flat blob stream dequantised in one pass: out[i] = act(act(code_i - 2^(b-1)) *
 * act(scale[i / group_size])), act = out_dtype (bf16 / fp16 / fp32).
 * Replaces vaayu/moe_patch.py:750-791 `_fused_dequant_kernel` / `_fused_dequant_fn`, the body
 * of `dequantize_expert_blob` (:849-864).  bits in {2, 4, 8}; group_size a multiple of 32/bits.
 */
int vy_dequant_flat(const int32_t* packed, int64_t n_words, int32_t bits, const void* scale,
                    int32_t scale_dtype, int32_t group_size, void* out, int32_t out_dtype,
                    void* stream);

/*
 * One projection [rows, cols] dequantised: out[r, c] = act(act(u - z) * act(scale[r, c / gs])),
 * z = 2^(b-1) when `zero` is NULL (the reference's symmetric format), else the stored zero code
 * of compressed-tensors' row-packed zero points zero[ceil(rows*b/32), cols/gs].
 * Replaces vaayu/moe_patch.py:713-744 `dequantize_packed_weight`; the zero-point form is an
 * extension (the reference refuses it, :724-729).
 */
int vy_dequant_packed_weight(const int32_t* packed, int64_t rows, int64_t cols, int32_t bits,
                             const void* scale, int32_t scale_dtype, int32_t group_size,
                             const int32_t* zero, void* out, int32_t out_dtype, void* stream);

/* ── block-scaled FP8 / FP4 ────────────────────────────────────────────────────────────── */

/*
 * out[r, c] = out_dtype(float(w[r, c]) * float(scale[r / bo, c / bi])), bo = rows / srows,
 * bi = cols / scols; w e4m3, scale fp32 / bf16 / e8m0.
 * Replaces vaayu/model_code/deepseek_v4/modeling_deepseek_v4.py:228-240 `dequantize_block_scaled`.
 */
int vy_fp8_dequant(const uint8_t* w, int64_t rows, int64_t cols, const void* scale,
                   int32_t scale_dtype, int64_t srows, int64_t scols, void* out,
                   int32_t out_dtype, void* stream);

/*
 * NVFP4: w [rows, cols/2] bytes holding two e2m1 codes (low nibble = even column), scale
 * [rows, cols/group_size] e4m3; out[r, c] = out_dtype(e2m1 * float(scale)).
 * No reference function (the nearest is the checkpoint-shipped fp4 GEMM behind
 * modeling_deepseek_v4.py:315-323, 353-363); the e2m1 table is the OCP MX one.
 */
int vy_fp4_dequant(const uint8_t* w, int64_t rows, int64_t cols, const uint8_t* scale,
                   int32_t group_size, void* out, int32_t out_dtype, void* stream);

/*
 * Dequant fused into a decode GEMV: out[t, n] = bf16(sum_k deq(W)[n, k] * x[t, k]), fp32
 * accumulation, x [n_tokens, k] bf16 (row stride x_stride), out [n_tokens, n] bf16 (row
 * stride out_stride), n_tokens <= 16.  The dequantised weight is exactly what vy_fp8_dequant /
 * vy_fp4_dequant produce.  No reference function: the reference dequantises at load
 * (modeling_deepseek_v4.py:243-270) and multiplies in bf16.
 */
int vy_fp8_gemv(const uint8_t* w, int64_t n, int64_t k, const void* scale, int32_t scale_dtype,
                int64_t srows, int64_t scols, const void* x, int64_t x_stride,
                int64_t n_tokens, void* out, int64_t out_stride, void* stream);
int vy_fp4_gemv(const uint8_t* w, int64_t n, int64_t k, const uint8_t* scale,
                int32_t group_size, const void* x, int64_t x_stride, int64_t n_tokens,
                void* out, int64_t out_stride, void* stream);

/* ── routing ───────────────────────────────────────────────────────────────────────────── */

/*
 * softmax(fp32 logits) -> top-k -> renormalised weights: weights [n_tokens, top_k] fp32,
 * ids [n_tokens, top_k] int64, largest first (ties to the lower expert id).
 * Replaces the fallback branch of vaayu/moe_patch.py:130-167 `route_experts` (:160-161) and of
 * `_route` (:2331-2334).  logits [n_tokens, n_experts] in logit_dtype, row stride.
 */
int vy_moe_topk_softmax(const void* logits, int32_t logit_dtype, int64_t row_stride,
                        int64_t n_tokens, int32_t n_experts, int32_t top_k, float* weights,
                        int64_t* ids, void* stream);

/*
 * Routed gather/permute plan, on the device (no host sync): the rows (token * top_k + slot)
 * grouped by expert id -- stable, ascending id -- and each token's slots in ascending expert id.
 *   order       [n_tokens*top_k]  row ids, each expert's rows a contiguous run in row order
 *   live_expert [n_experts]       the routed expert ids, ascending; entries >= n_live unused
 *   live_start  [n_experts+1]     live_start[i] = first position of live_expert[i] in `order`
 *   slot_order  [n_tokens*top_k]  row ids of token t's slots, ascending expert id then slot
 *   counters    [4]               n_live, rows dropped for an out-of-range id, 0, 0
 * Replaces vaayu/packed_expert_kernels.py:676-717 `_prefill_plan` / `_prefill_tables` (host
 * argsort + pinned upload) and vaayu/moe_patch.py:306-326 `compute_expert_dispatch`.
 * ids [n_tokens, top_k] contiguous, ids_dtype VY_I32 or VY_I64.  n_experts <= 1024.
 */
int vy_moe_route_permute(const void* ids, int32_t ids_dtype, int64_t n_tokens, int32_t top_k,
                         int32_t n_experts, int32_t* order, int32_t* live_expert,
                         int32_t* live_start, int32_t* slot_order, int32_t* counters,
                         void* stream);

/* ── the fused expert layer ────────────────────────────────────────────────────────────── */

/*
 * Geometry of one expert blob (`build_expert_blob`, vaayu/moe_patch.py:794-846): three
 * projections gate [inter, hidden], up [inter, hidden], down [hidden, inter] packed along K in
 * one int32 stream, one scale stream and (optionally) one row-packed zero-point stream.  The
 * offsets say where each role starts inside its stream (index 0 gate, 1 up, 2 down), so any
 * role order is accepted (the reference's blobs are ordered gate, down, up).
 */
typedef struct vy_expert_geom {
    int32_t hidden;
    int32_t inter;
    int32_t bits;         /* 4 */
    int32_t group_size;   /* power of two >= 32, dividing hidden and inter */
    int32_t scale_dtype;  /* VY_BF16 / VY_F16 / VY_F32 */
    int32_t has_zero;     /* 0: symmetric (zero 2^(b-1)), 1: zero-point stream present */
    int64_t word_off[3];
    int64_t scale_off[3];
    int64_t zero_off[3];
} vy_expert_geom;

/*
 * One MoE layer call.  Row j = t * top_k + k is slot k of token t; it routes to expert
 * expert_ids[j] (an index into expert_table) with weight
 *   weights[t * w_tok_stride + (w_index ? w_index[j] : k) * w_slot_stride].
 * expert_table[e] = {packed stream, scale stream, zero stream (or 0)} device addresses of
 * expert e's blob (int64 each).  Per row: g = act(x.Wg), u = act(x.Wu), a = act(silu(g)),
 * h = act(a * u), y = act(h.Wd), c = fp32(y) * w (rounded to act when w_dtype == act_dtype),
 * and out[t] = the fp32 sum of token t's c in ascending expert index, then slot
 * (vaayu/moe_patch.py:914-940).  `out` is overwritten.  When `contrib` is non-NULL the per-row
 * c go there ([n_tokens*top_k, hidden] fp32) and `out` is not written (the expert-parallel
 * combine sums them on the token's home rank).  `h_out` (optional, [n_tokens*top_k, inter],
 * act dtype) receives each row's h: a stage probe for tests.
 *
 * Fields appended in ABI version 2 (zero keeps version-1 behaviour):
 *   col_blocks      tokens one decode pass of an expert carries, in blocks of 8: 1, 2 or 4 (0:
 *                   chosen by the library: 2 for at most 16 experts with at most 4 routed rows
 *                   each on average, else 1).  An expert with more routed rows takes more passes
 *                   (its weights are read once per pass, the later ones mostly from L2).
 *   expert_base     expert_ids[j] - expert_base indexes expert_table; ids outside
 *                   [expert_base, expert_base + n_experts) drop their slot (a rank's own range of a
 *                   global id space).
 *   ids_row_stride  elements between consecutive tokens' rows of expert_ids (0: top_k).
 *
 * Fields appended in ABI version 3 (zero keeps version-2 behaviour):
 *   shared_last     1: slot top_k - 1 of every token is the block's always-on shared expert (an
 *                   entry of expert_table like any other, routed with weight 1 or its sigmoid
 *                   gate), and the layer ends with the model's epilogue
 *                     result[t] = act(act(sum of the routed slots' c) + act(c of the shared slot))
 *                   (vaayu/packed_expert_kernels.py:502-508: out.to(act) + shared.to(act)), the
 *                   routed sum in ascending expert index as above.  `out` (optional here)
 *                   receives that routed fp32 sum; `contrib` must be NULL.
 *   result          [n_tokens, hidden] act dtype, written when shared_last is 1.
 *   result_row_stride  elements between result rows (>= hidden).
 *   k_splits        decode: warps sharing one gate/up unit's K range -- 0: the library's choice
 *                   (more than one only when a call has few units per warp, e.g. 1-4 tokens),
 *                   1: none, 2 / 4 / 8: that many (dividing hidden / 128).  The result does not
 *                   depend on it (each unit's per-stage partials are added in stage order).
 */
typedef struct vy_moe_call {
    const vy_expert_geom* geom;
    int32_t act_dtype;        /* VY_BF16 or VY_F16 */
    int32_t n_experts;
    int32_t top_k;
    int32_t ids_dtype;        /* VY_I32 / VY_I64 */
    int64_t n_tokens;
    const void* x;            /* [n_tokens, hidden], act dtype */
    int64_t x_row_stride;
    const int64_t* expert_table;
    const void* expert_ids;   /* [n_tokens, top_k] contiguous */
    const void* weights;
    int32_t w_dtype;          /* VY_F32 / VY_BF16 / VY_F16 */
    int32_t reserved0;
    int64_t w_tok_stride;
    int64_t w_slot_stride;
    const int32_t* w_index;   /* optional */
    float* out;               /* [n_tokens, hidden] fp32 */
    int64_t out_row_stride;
    float* contrib;           /* optional */
    void* h_out;              /* optional */
    void* workspace;
    size_t workspace_bytes;
    /* Optional per-stage timing (the reference's per-phase profile, vaayu/moe_patch.py:2431-2438):
     * when non-NULL, n_stage_events (>= 4) cudaEvent_t handles recorded on `stream` before the
     * routing plan, after it (and, for prefill, the row gather), after the gate/up stage and after
     * the down/combine stage; vy_moe_prefill records a fifth, when given, between the down GEMM and
     * the combine.  Recording them serialises the stages (no programmatic overlap): a profiling
     * mode, not the fast path. */
    void* const* stage_events;
    int32_t n_stage_events;
    int32_t reserved1;
    /* ABI version 2 */
    int32_t col_blocks;
    int32_t expert_base;
    int64_t ids_row_stride;
    /* ABI version 3 */
    int32_t shared_last;
    int32_t k_splits;
    void* result;
    int64_t result_row_stride;
} vy_moe_call;

/*
 * out[i] = ((parts[0][i] + parts[1][i]) + ...) + parts[n_parts-1][i], fp32, in part order: the
 * expert-parallel combine of per-rank partial sums (ranks hold ascending expert ranges).  parts
 * is [n_parts][n] contiguous; n a multiple of 4, both pointers 16-byte aligned.  No counterpart
 * in the reference (it is single-GPU).
 */
int vy_sum_ordered(const float* parts, int32_t n_parts, int64_t n, float* out, void* stream);

/*
 * Expert-parallel dispatch plan: addresses each (token, slot) row j = t * top_k + k of this
 * rank's batch to the rank holding its expert and packs the send buffers of fixed-capacity,
 * equal-split all-to-alls (the exchange itself is the caller's: NCCL).  No counterpart in the
 * reference (it is single-GPU).
 *   ids [n_tokens, ids_row_stride]   GLOBAL expert ids (int32 / int64); an id outside
 *                                    [0, n_ranks * experts_per_rank) is dropped
 *   placement                        0: expert e on rank e / experts_per_rank as local expert
 *                                    e % experts_per_rank; 1 (interleaved): rank e % n_ranks,
 *                                    local e / n_ranks
 *   weights                          routing weights, element (t, k) at t * w_tok_stride +
 *                                    k * w_slot_stride (bf16 / fp16 / fp32)
 *   x [n_tokens, x_row_stride]       activations (bf16 / fp16), hidden columns used
 *   capacity                         slots per destination; n_tokens * top_k takes any routing
 * Row j takes slot dest * capacity + pos, pos its rank among the rows bound for dest, in row
 * order; a row past a full destination is dropped.  Outputs (device memory):
 *   send_ids [n_ranks * capacity]    int32 local expert id; -1 for an empty slot
 *   send_w   [n_ranks * capacity]    fp32 routing weight
 *   send_x   [n_ranks * capacity, hidden] the token's activations (empty slots unwritten)
 *   slot_of_row [n_tokens * top_k]   int64 slot, -1 for a dropped row
 *   counts   [n_ranks]               int32 rows taken per destination
 *   wanted   [n_ranks]               optional (NULL: not written): int32 rows bound for each
 *                                    destination before the capacity cut; a caller that sizes
 *                                    `capacity` below n_tokens * top_k detects a dropped row as
 *                                    wanted[d] > capacity (appended in ABI version 4)
 */
int vy_ep_dispatch_plan(const void* ids, int32_t ids_dtype, int64_t ids_row_stride, int64_t n_tokens,
                        int32_t top_k, int32_t n_ranks, int32_t experts_per_rank, int32_t placement,
                        const void* weights, int32_t w_dtype, int64_t w_tok_stride, int64_t w_slot_stride,
                        const void* x, int32_t x_dtype, int64_t x_row_stride, int64_t hidden,
                        int64_t capacity, int32_t* send_ids, float* send_w, void* send_x,
                        int64_t* slot_of_row, int32_t* counts, int32_t* wanted, void* stream);

/*
 * Expert-parallel combine on the tokens' home rank: out[t] = sum over token t's slots, in
 * ascending GLOBAL expert id then slot (fp32), of back[slot_of_row[t * top_k + k]] -- the
 * contributions returned by the reverse all-to-all, read in place through the dispatch plan's
 * slot map (-1: none).  The order `accumulate_expert_outputs` (vaayu/moe_patch.py:914-940)
 * sums in, so the result equals one GPU's layer bit for bit.  expert_ids [n_tokens,
 * ids_row_stride] (0: top_k, contiguous) -- the same ids, with the same stride, as the dispatch
 * plan was given (ids_row_stride appended in ABI version 4).  n_tokens <= 65535.
 */
int vy_ep_combine(const float* back, const int64_t* slot_of_row, const void* expert_ids, int32_t ids_dtype,
                  int64_t ids_row_stride, int64_t n_tokens, int32_t top_k, int64_t hidden, float* out,
                  int64_t out_row_stride, void* stream);

/*
 * Error flags of the last vy_moe_decode (path 0) / vy_moe_prefill (path 1) call made with this
 * call structure and workspace, copied (enqueued on `stream`) to `out` (device or host int32):
 *   VY_FLAG_BAD_EXPERT  a routed expert's streams were unusable (null or misaligned pointer);
 *                       its slots contributed nothing
 *   VY_FLAG_TIMEOUT     a device-side barrier wait ran out (bounded, never a hang); the work item
 *                       it belonged to was abandoned and its output is not valid
 *   VY_FLAG_DRAIN       draining in-flight copies after such a timeout ran out as well
 * 0 = clean.  The routing plan of every call clears them.  For a vy_moe_decode_static call, pass
 * the same call structure with workspace NULL and path 0: the flags are read from the library's
 * scratch array (they are the last static call's, on the current device).  No counterpart in the
 * reference.
 */
#define VY_FLAG_BAD_EXPERT 1
#define VY_FLAG_TIMEOUT 4
#define VY_FLAG_DRAIN 8
int vy_moe_error_flags(const vy_moe_call* call, int32_t path, int32_t* out, void* stream);

/*
 * Self-test of the failure path: one CTA runs the kernels' bounded barrier wait on a barrier that
 * expects two arrivals and gets `arrivals` (0-2).  With fewer than two the wait gives up after
 * `limit_ns` (<= 2 s) and ORs VY_FLAG_TIMEOUT into *flags (device int32); the context stays usable.
 */
int vy_selftest_bounded_wait(int32_t arrivals, int64_t limit_ns, int32_t* flags, void* stream);

/* Bytes of workspace vy_moe_decode (path 0) / vy_moe_prefill (path 1) need for `call`.  For a
 * decode call with k_splits = 0 this includes the split-K partials a few-token call may use; a
 * workspace of at least the k_splits = 1 size is accepted too (the call then runs unsplit, with
 * the same result), so one workspace sized for the largest batch serves every smaller one. */
size_t vy_moe_workspace_size(const vy_moe_call* call, int32_t path);

/*
 * The layer through the bandwidth-bound kernels: a token-batched dequant GEMV that reads each
 * routed expert's packed weights once for all its tokens.  For decode-sized calls.
 * Replaces vaayu/packed_expert_kernels.py:130-176 `_gate_up_kernel` / `_down_kernel` and their
 * launcher `_launch` (:390-396) behind `packed_experts_decode` (:459-480).
 */
int vy_moe_decode(const vy_moe_call* call, void* stream);

/*
 * The layer through the tensor-core grouped GEMM (tcgen05, accumulators in TMEM): int4
 * dequantised into shared memory, 128-row tiles per expert.  For prefill-sized calls.
 * Replaces vaayu/packed_expert_kernels.py:178-260 `_gate_up_grouped` / `_down_grouped` /
 * `_reduce_kernel` and `_prefill_launch` (:760-777) behind `packed_experts_prefill` (:838-861).
 */
int vy_moe_prefill(const vy_moe_call* call, void* stream);

/*
 * Bytes of the scratch array compiled into the library for vy_moe_decode_static.  Every GPU that
 * loads the library holds this much device memory until the process exits.  Sized for the
 * split-K partials of a two-token call at top-k 8 on a 2048 x 768 layer (about 15 MB).
 */
#define VY_DECODE_STATIC_SCRATCH_BYTES (16u << 20)

/*
 * vy_moe_decode with no workspace from the caller and no allocation: the scratch is a fixed array
 * of VY_DECODE_STATIC_SCRATCH_BYTES inside the library (call->workspace and workspace_bytes are
 * ignored).  This entry point has no counterpart in the reference.  It is for hosts that cannot
 * call cudaMalloc -- a binding that only receives pointers from a runtime owning all device
 * memory, an engine whose memory plan has no room left, code that must not allocate while it runs
 * -- and so cannot supply vy_moe_decode's workspace.  A call whose vy_moe_workspace_size (path 0)
 * exceeds the array is rejected with VY_ERR_UNSUPPORTED.  The first call on each device looks the
 * array's device address up (once, with that device current); make that first call before any
 * stream capture.  All calls share the array: calls whose kernels overlap on the GPU race on it
 * and must be ordered on one stream.  Results are bit-identical to vy_moe_decode's.
 */
int vy_moe_decode_static(const vy_moe_call* call, void* stream);

/*
 * out[t] = sum of contrib[t * top_k + k] over the token's slots in ascending expert id, then
 * slot (fp32), for contributions gathered back from other ranks.  Replaces
 * vaayu/packed_expert_kernels.py:249-260 `_reduce_kernel` with the order
 * `accumulate_expert_outputs` (vaayu/moe_patch.py:914-940) sums in.
 */
int vy_moe_combine(const float* contrib, const void* expert_ids, int32_t ids_dtype,
                   int64_t n_tokens, int32_t top_k, int64_t hidden, float* out,
                   int64_t out_row_stride, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* VAAYU_B200_H */
