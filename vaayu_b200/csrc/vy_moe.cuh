// vy_moe.cuh -- internal interfaces between the routing, decode and prefill translation units.
#pragma once

#include "vy_common.cuh"

namespace vy {

constexpr int kMaxTopK = 32;
constexpr int kMaxExperts = 1024;
constexpr int kMaxPassCols = 32;   // tokens one pass of an expert carries (8 per column block)

// One pass of one live expert: the unit of work of the GEMV kernels, fully resolved by the
// routing plan so a kernel fetches it with independent loads (no dependent pointer chase).
struct __align__(16) PassEntry {
    int64_t pk, sc, zp;            // the expert's packed / scale / zero streams
    int32_t row0;                  // first position of this pass in `order`
    int32_t ncols;                 // routed rows in this pass (<= tok_per_unit)
    int32_t rows[kMaxPassCols];    // their row ids (token * top_k + slot)
};

// Arguments of the routing plan kernel (block 0) and the activation permutation (blocks >= 1).
struct PlanArgs {
    const void* ids;
    bool ids64;
    int64_t ids_stride;    // elements between tokens' id rows (top_k when contiguous)
    int id_base;           // ids are offset by this (a rank's range of a global id space)
    int64_t n_tokens;
    int top_k;
    int n_experts;
    int32_t* order;        // [n]       row ids grouped by expert (stable)
    int32_t* live_expert;  // [E]       routed expert ids ascending
    int32_t* live_start;   // [E+1]     start of each live expert's run in `order`
    int32_t* unit_start;   // [E+1]     optional: prefix of ceil(count / tok_per_unit)
    int32_t* slot_order;   // [n]       token t's row ids, ascending expert id then slot
    int32_t* counters;     // [4]       n_live, dropped rows, kernel error flags, spare
    int tok_per_unit;
    // activation permutation (x -> x_perm, 8-element groups), skipped when x_perm is null
    const void* x;
    int64_t x_stride;
    bool x_vec;
    int64_t hidden;
    uint16_t* x_perm;
    // an int array the plan zeroes before anything else of the call runs (per-tile tickets)
    int32_t* zero_ints;
    int zero_count;
    // optional pass table (needs unit_start and tok_per_unit): one PassEntry per expert pass
    const int64_t* expert_table;
    PassEntry* passes;
};

size_t plan_smem_bytes(int n_experts);
int plan_validate(int64_t n_tokens, int top_k, int n_experts);
int launch_plan(const PlanArgs& p, int sm_count, cudaStream_t stream);
// out[t] = sum of contrib rows slot_order[t*top_k .. +top_k) (row ids, -1 = none), fp32, in
// that order; launched with programmatic stream serialisation.
int launch_slot_combine(const float* contrib, const int32_t* slot_order, int64_t n_tokens, int top_k, int hidden,
                        float* out, int64_t out_stride, cudaStream_t s);
// A layer call's final combine: launch_slot_combine, or with c->shared_last the shared-expert
// epilogue into c->result (and the routed sum into c->out when given).
int launch_layer_combine(const vy_moe_call* c, const float* contrib, const int32_t* slot_order, cudaStream_t s);
// out[t] = sum over token t's slots, ascending expert id then slot, of contribution row
// t * top_k + k -- or rows[t * top_k + k] when `rows` is given (-1: no contribution).  Token t's
// ids start at ids[t * ids_stride] (0: top_k, contiguous).
// `chained`: launched with programmatic stream serialisation (it waits for the previous kernel).
int launch_combine(const float* contrib, const void* ids, bool ids64, int64_t n_tokens,
                   int top_k, int64_t hidden, float* out, int64_t out_stride, int sm_count,
                   cudaStream_t stream, const int64_t* rows = nullptr, int64_t ids_stride = 0,
                   bool chained = false);

// Shared validation of a vy_moe_call (decode and prefill entry points).
int validate_call(const vy_moe_call* c);
size_t prefill_workspace_bytes(const vy_moe_call* c);
int32_t* prefill_flags(const vy_moe_call* c);   // the call's error flags in its (prefill) workspace
// The device address of the scratch array vy_moe_decode_static uses, on the current device.
int decode_static_scratch(void** out);

// Workspace carve-up shared by the decode and prefill entry points.
struct Carve {
    char* base;
    size_t used;
    template <typename T>
    T* take(size_t count) {
        size_t off = (used + 255) & ~size_t(255);
        used = off + count * sizeof(T);
        return base ? reinterpret_cast<T*>(base + off) : nullptr;
    }
};

}  // namespace vy
