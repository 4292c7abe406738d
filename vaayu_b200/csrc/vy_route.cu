// vy_route.cu -- routing on the device: softmax top-k, the routed gather/permute plan (a
// stable counting sort of (token, slot) rows by expert id), the activation permutation the
// GEMV kernels read, and the ordered weighted combine.
#include <climits>

#include "vy_moe.cuh"

namespace vy {
namespace {

constexpr int kPlanThreads = 1024;
constexpr int kPlanWarps = kPlanThreads / 32;

__device__ __forceinline__ int load_id(const void* ids, bool ids64, int64_t j) {
    if (ids64) {
        int64_t v = reinterpret_cast<const int64_t*>(ids)[j];
        return (v < INT32_MIN || v > INT32_MAX) ? -1 : static_cast<int>(v);
    }
    return reinterpret_cast<const int32_t*>(ids)[j];
}

// Expert index of row j = t * top_k + k (id - id_base; the caller range-checks it).
__device__ __forceinline__ int plan_id(const PlanArgs& p, int64_t j) {
    int64_t idx = j;
    if (p.ids_stride != p.top_k) {
        const int64_t t = j / p.top_k;
        idx = t * p.ids_stride + (j - t * p.top_k);
    }
    const int e = load_id(p.ids, p.ids64, idx);
    return e < 0 ? -1 : e - p.id_base;
}

// Exclusive scan of one int per thread over the block (any whole number of warps up to
// kPlanWarps); returns this thread's prefix and puts the total in *total.  `scratch` holds
// kPlanWarps + 1 ints.
__device__ int block_exclusive_scan(int v, int* scratch, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) scratch[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = lane < nw ? scratch[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < nw) scratch[lane] = w;   // inclusive prefix of warp sums
        if (lane == nw - 1) scratch[kPlanWarps] = w;
    }
    __syncthreads();
    int base = warp > 0 ? scratch[warp - 1] : 0;
    *total = scratch[kPlanWarps];
    int excl = base + x - v;
    __syncthreads();
    return excl;
}

// The plan of a decode-sized call (n <= kSmallPlan rows): a bitonic sort of the keys
// (expert id << 10 | row) -- unique, so the sort is stable by construction -- with warp shuffles
// for the exchanges inside a warp and shared memory above that, then the run boundaries of the
// sorted keys give the live experts.  n <= 32 stays in one warp with no barrier at all.
constexpr int kSmallPlan = kPlanThreads;
constexpr int kKeyNone = 0x7FFFFFFF;

__device__ __forceinline__ int warp_sort_step(int key, int lane_id, int k, int j) {
    const int other = __shfl_xor_sync(0xffffffffu, key, j);
    const bool up = (lane_id & k) == 0, lower = (lane_id & j) == 0;
    return (lower == up) ? min(key, other) : max(key, other);
}

// Each row's place among its token's slots (ascending id, then slot; dropped rows last).
__device__ __forceinline__ void write_slot_order(const PlanArgs& p, const int* ids, int j, int n) {
    if (j >= n) return;
    const int K = p.top_k, t = j / K, k = j - t * K, e = ids[j];
    int pos = 0;
    for (int q = 0; q < K; ++q) {
        const int v = ids[t * K + q];
        pos += (e >= 0) ? (v >= 0 && (v < e || (v == e && q < k))) : (v >= 0 || q < k);
    }
    p.slot_order[t * K + pos] = e >= 0 ? j : -1;
}

// Sorted position `pos` of a live expert's run (run start `ls`, length `count`, first pass
// `ustart`, expert `e`) holds row `row`: file it in the pass table.
__device__ __forceinline__ void file_pass_row(const PlanArgs& p, const int64_t* table, int e, int ls, int count,
                                              int ustart, int pos, int row) {
    if (!p.passes) return;
    const int tpu = p.tok_per_unit, r = pos - ls, q = r / tpu, col = r - q * tpu;
    PassEntry& pe = p.passes[ustart + q];
    if (col < kMaxPassCols) pe.rows[col] = row;   // row ids are kept for GEMV-sized passes only
    if (col == 0) {
        pe.pk = table[3 * e];
        pe.sc = table[3 * e + 1];
        pe.zp = table[3 * e + 2];
        pe.row0 = pos;
        pe.ncols = min(tpu, count - q * tpu);
    }
}

__device__ void plan_small(const PlanArgs& p) {
    __shared__ int ids[kSmallPlan];
    __shared__ int keys[kSmallPlan];
    __shared__ int ls[kSmallPlan + 1];
    __shared__ int scratch[kPlanWarps + 1];
    __shared__ int64_t table[3 * kMaxExperts];   // the expert pointer table, read while sorting
    const int n = static_cast<int>(p.n_tokens * p.top_k), tid = threadIdx.x, E = p.n_experts;
    const int lane = tid & 31;
    if (p.passes)
        for (int i = tid; i < 3 * E; i += blockDim.x) table[i] = p.expert_table[i];
    int e = -1;
    if (tid < n) {
        e = plan_id(p, tid);
        if (e < 0 || e >= E) e = -1;
        ids[tid] = e;
    }
    int key = (tid < n && e >= 0) ? ((e << 10) | tid) : kKeyNone;
    const int tpu = p.tok_per_unit;
    if (n <= 32) {
        __syncthreads();                         // ids[] and table[] in place
        if (tid >= 32) return;
        for (int k = 2; k <= 32; k <<= 1)
            for (int j = k >> 1; j > 0; j >>= 1) key = warp_sort_step(key, lane, k, j);
        const bool valid = key != kKeyNone;
        const int ek = valid ? (key >> 10) : -1;
        const int prev = __shfl_up_sync(0xffffffffu, ek, 1);
        const bool first = valid && (lane == 0 || prev != ek);
        const unsigned fm = __ballot_sync(0xffffffffu, first);
        const int n_valid = __popc(__ballot_sync(0xffffffffu, valid));
        const int li = __popc(fm & ((1u << lane) - 1u));
        // run end = next first position (or n_valid); units prefix over the live runs
        const unsigned later = fm & ~((2u << lane) - 1u);
        const int run_end = later ? (__ffs(later) - 1) : n_valid;
        int units = (first && tpu > 0) ? (run_end - lane + tpu - 1) / tpu : 0;
        int incl = units;
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        if (valid) p.order[lane] = key & 1023;
        if (first) {
            p.live_expert[li] = ek;
            p.live_start[li] = lane;
            if (p.unit_start) p.unit_start[li] = incl - units;
        }
        if (p.passes) {
            // every position learns its run: the start (last first-flag at or before it)
            const unsigned upto = fm & ((2u << lane) - 1u);
            const int run_start = valid ? (31 - __clz(upto)) : 0;
            const int rend = __shfl_sync(0xffffffffu, run_end, run_start);
            const int ust = __shfl_sync(0xffffffffu, incl - units, run_start);
            if (valid) file_pass_row(p, table, ek, run_start, rend - run_start, ust, lane, key & 1023);
        }
        const int n_live = __popc(fm), total_units = __shfl_sync(0xffffffffu, incl, 31);
        if (lane == 0) {
            p.live_start[n_live] = n_valid;
            if (p.unit_start) p.unit_start[n_live] = total_units;
            p.counters[0] = n_live;
            p.counters[1] = n - n_valid;
            p.counters[2] = 0;
            p.counters[3] = 0;
        }
        write_slot_order(p, ids, lane, n);
        return;
    }
    // block-wide bitonic sort over the next power of two >= n
    int N = 64;
    while (N < n) N <<= 1;
    for (int k = 2; k <= N; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            if (j >= 32) {
                keys[tid] = key;
                __syncthreads();
                const int other = keys[tid ^ j];
                __syncthreads();
                const bool up = (tid & k) == 0, lower = (tid & j) == 0;
                key = (lower == up) ? min(key, other) : max(key, other);
            } else {
                key = warp_sort_step(key, tid, k, j);
            }
        }
    }
    keys[tid] = key;
    __syncthreads();
    const bool valid = tid < N && key != kKeyNone;
    const int ek = valid ? (key >> 10) : -1;
    const bool first = valid && (tid == 0 || (keys[tid - 1] >> 10) != ek);
    int n_live, n_valid;
    const int li = block_exclusive_scan(first ? 1 : 0, scratch, &n_live);
    block_exclusive_scan(valid ? 1 : 0, scratch, &n_valid);
    if (valid) p.order[tid] = key & 1023;
    if (first) {
        p.live_expert[li] = ek;
        ls[li] = tid;
    }
    if (tid == 0) ls[n_live] = n_valid;
    __syncthreads();
    const int units = (tid < n_live && tpu > 0) ? (ls[tid + 1] - ls[tid] + tpu - 1) / tpu : 0;
    int total_units;
    const int ustart = block_exclusive_scan(units, scratch, &total_units);
    if (tid <= n_live) {
        p.live_start[tid] = ls[tid];
        if (p.unit_start) p.unit_start[tid] = tid < n_live ? ustart : total_units;
    }
    if (p.passes) {
        keys[tid] = ustart;                       // keys[] is free now: per-live-expert first pass
        __syncthreads();
        const int run = li + (first ? 1 : 0) - 1; // this position's live index
        if (valid) file_pass_row(p, table, ek, ls[run], ls[run + 1] - ls[run], keys[run], tid, key & 1023);
    }
    if (tid == 0) {
        p.counters[0] = n_live;
        p.counters[1] = n - n_valid;
        p.counters[2] = 0;
        p.counters[3] = 0;
    }
    write_slot_order(p, ids, tid, n);
}

// Block 0: the plan.  Blocks >= 1: the activation permutation (x -> x_perm).
__global__ void __launch_bounds__(kPlanThreads) plan_kernel(PlanArgs p) {
    // launched with programmatic serialisation: the previous kernel on the stream (often the last
    // call's combine) may still run; nothing here reads or writes before it has completed
    grid_dependency_wait();
    grid_dependents_launch();   // the gate/up grid may be scheduled now; it waits for this grid
    if (blockIdx.x > 0) {
        // each thread permutes one 8-element group of one token's activations
        const int64_t groups_per_tok = p.hidden / 8;
        const int64_t total = p.n_tokens * groups_per_tok;
        for (int64_t q = (blockIdx.x - 1) * int64_t(blockDim.x) + threadIdx.x; q < total;
             q += int64_t(gridDim.x - 1) * blockDim.x) {
            const int64_t t = q / groups_per_tok, c = (q % groups_per_tok) * 8;
            const uint16_t* src = reinterpret_cast<const uint16_t*>(p.x) + t * p.x_stride + c;
            uint16_t v[8];
            if (p.x_vec) {
                *reinterpret_cast<uint4*>(v) = *reinterpret_cast<const uint4*>(src);
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = src[j];
            }
            uint4 o;
            o.x = v[0] | (uint32_t(v[4]) << 16);
            o.y = v[1] | (uint32_t(v[5]) << 16);
            o.z = v[2] | (uint32_t(v[6]) << 16);
            o.w = v[3] | (uint32_t(v[7]) << 16);
            *reinterpret_cast<uint4*>(p.x_perm + t * p.hidden + c) = o;
        }
        return;
    }
    for (int i = threadIdx.x; i < p.zero_count; i += blockDim.x) p.zero_ints[i] = 0;
    const int64_t n_rows_all = p.n_tokens * p.top_k;
    if (n_rows_all <= kSmallPlan) {
        plan_small(p);
        return;
    }
    extern __shared__ int cnt[];                            // [kPlanWarps][n_experts]
    __shared__ int scan_scratch[kPlanWarps + 1];
    __shared__ int dropped;
    const int E = p.n_experts, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t n = p.n_tokens * p.top_k;
    const int64_t seg = (n + kPlanWarps - 1) / kPlanWarps;
    const int64_t lo = warp * seg, hi = min(n, lo + seg);
    int* my = cnt + warp * E;
    if (threadIdx.x == 0) dropped = 0;
    for (int e = lane; e < E; e += 32) my[e] = 0;
    __syncthreads();
    // 1. per-warp histogram of its contiguous segment of rows
    for (int64_t base = lo; base < hi; base += 32) {
        const int64_t row = base + lane;
        int e = -1;
        if (row < hi) {
            e = plan_id(p, row);
            if (e < 0 || e >= E) {
                atomicAdd(&dropped, 1);
                e = -1;
            }
        }
        const unsigned mask = __match_any_sync(0xffffffffu, e);
        if (e >= 0 && lane == __ffs(mask) - 1) my[e] += __popc(mask);
        __syncwarp();
    }
    __syncthreads();
    // 2. totals, expert starts, the live list, unit prefix; per-warp counts become each
    //    warp's first position inside the expert's run (warp order = row order: stable)
    const int e = threadIdx.x;
    int tot = 0;
    if (e < E)
        for (int w = 0; w < kPlanWarps; ++w) tot += cnt[w * E + e];
    int n_rows, n_live, n_units;
    const int start = block_exclusive_scan(tot, scan_scratch, &n_rows);
    const int live_idx = block_exclusive_scan(tot > 0 ? 1 : 0, scan_scratch, &n_live);
    const int units = (tot > 0 && p.tok_per_unit > 0) ? (tot + p.tok_per_unit - 1) / p.tok_per_unit : 0;
    const int ustart = block_exclusive_scan(units, scan_scratch, &n_units);
    if (e < E) {
        if (tot > 0) {
            p.live_expert[live_idx] = e;
            p.live_start[live_idx] = start;
            if (p.unit_start) p.unit_start[live_idx] = ustart;
        }
        int running = start;
        for (int w = 0; w < kPlanWarps; ++w) {
            const int c = cnt[w * E + e];
            cnt[w * E + e] = running;
            running += c;
        }
    }
    if (threadIdx.x == 0) {
        p.live_start[n_live] = n_rows;
        if (p.unit_start) p.unit_start[n_live] = n_units;
        p.counters[0] = n_live;
        p.counters[1] = dropped;
        p.counters[2] = 0;
        p.counters[3] = 0;
    }
    __syncthreads();
    // 3. stable scatter: position = warp's next slot for the id + rank among equal ids
    for (int64_t base = lo; base < hi; base += 32) {
        const int64_t row = base + lane;
        int ex = -1;
        if (row < hi) {
            ex = plan_id(p, row);
            if (ex < 0 || ex >= E) ex = -1;
        }
        const unsigned mask = __match_any_sync(0xffffffffu, ex);
        int pos = 0;
        if (ex >= 0) pos = my[ex] + __popc(mask & ((1u << lane) - 1u));
        __syncwarp();
        if (ex >= 0) {
            p.order[pos] = static_cast<int32_t>(row);
            if (lane == __ffs(mask) - 1) my[ex] += __popc(mask);
        }
        __syncwarp();
    }
    // 3b. the pass table: each sorted position finds its live run by binary search
    if (p.passes) {
        __syncthreads();
        __threadfence_block();
        for (int64_t pos = threadIdx.x; pos < n_rows; pos += blockDim.x) {
            int lo = 0, hi = n_live - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (p.live_start[mid] <= pos) lo = mid;
                else hi = mid - 1;
            }
            const int ls0 = p.live_start[lo];
            file_pass_row(p, p.expert_table, p.live_expert[lo], ls0, p.live_start[lo + 1] - ls0, p.unit_start[lo],
                          static_cast<int>(pos), p.order[pos]);
        }
    }
    // 4. each token's slots in ascending expert id (stable by slot); dropped slots last as -1
    const int K = p.top_k;
    for (int64_t t = threadIdx.x; t < p.n_tokens; t += blockDim.x) {
        int key[kMaxTopK], idx[kMaxTopK];
        for (int k = 0; k < K; ++k) {
            int ex = plan_id(p, t * K + k);
            key[k] = (ex < 0 || ex >= E) ? INT32_MAX : ex;
            idx[k] = k;
        }
        for (int a = 1; a < K; ++a) {
            int kv = key[a], iv = idx[a], b = a - 1;
            while (b >= 0 && key[b] > kv) {
                key[b + 1] = key[b];
                idx[b + 1] = idx[b];
                --b;
            }
            key[b + 1] = kv;
            idx[b + 1] = iv;
        }
        for (int k = 0; k < K; ++k)
            p.slot_order[t * K + k] = key[k] == INT32_MAX ? -1 : static_cast<int32_t>(t * K + idx[k]);
    }
}

// softmax -> top-k -> renormalise; one warp per token.
template <int LD>
__global__ void topk_softmax_kernel(const void* logits, int64_t row_stride, int64_t n_tokens,
                                    int n_experts, int top_k, float* weights, int64_t* ids) {
    const int lane = threadIdx.x & 31;
    const int64_t t = blockIdx.x * int64_t(blockDim.x / 32) + (threadIdx.x >> 5);
    if (t >= n_tokens) return;
    auto val = [&](int e) -> float {
        if constexpr (LD == VY_F32) return reinterpret_cast<const float*>(logits)[t * row_stride + e];
        else if constexpr (LD == VY_BF16)
            return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(logits)[t * row_stride + e]);
        else return __half2float(reinterpret_cast<const __half*>(logits)[t * row_stride + e]);
    };
    float mx = -INFINITY;
    for (int e = lane; e < n_experts; e += 32) mx = fmaxf(mx, val(e));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
    for (int e = lane; e < n_experts; e += 32) sum += expf(val(e) - mx);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    // top-k by repeated arg-max over the probabilities (largest first, ties to the lower id)
    float chosen_p[kMaxTopK];
    int chosen_e[kMaxTopK];
    float ksum = 0.f;
    for (int k = 0; k < top_k; ++k) {
        float best = -1.f;
        int be = INT32_MAX;
        for (int e = lane; e < n_experts; e += 32) {
            bool taken = false;
            for (int q = 0; q < k; ++q) taken |= (chosen_e[q] == e);
            if (taken) continue;
            float pv = expf(val(e) - mx) / sum;
            if (pv > best || (pv == best && e < be)) {
                best = pv;
                be = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float ob = __shfl_xor_sync(0xffffffffu, best, o);
            int oe = __shfl_xor_sync(0xffffffffu, be, o);
            if (ob > best || (ob == best && oe < be)) {
                best = ob;
                be = oe;
            }
        }
        chosen_p[k] = best;
        chosen_e[k] = be;
    }
    for (int k = 0; k < top_k; ++k) ksum += chosen_p[k];
    if (lane == 0) {
        for (int k = 0; k < top_k; ++k) {
            weights[t * top_k + k] = chosen_p[k] / ksum;
            ids[t * top_k + k] = chosen_e[k];
        }
    }
}

// out[t] = sum of contrib rows of token t in slot_order (ascending expert id, then slot).
__global__ void combine_kernel(const float* __restrict__ contrib, const void* ids, bool ids64,
                               int64_t ids_stride, int64_t n_tokens, int top_k, int64_t hidden, float* out,
                               int64_t out_stride, const int64_t* __restrict__ rows) {
    grid_dependency_wait();      // when launched chained: the contributions' producer has finished
    const int64_t t = blockIdx.y;
    int idx[kMaxTopK];
    int key[kMaxTopK];
    for (int k = 0; k < top_k; ++k) {
        int e = load_id(ids, ids64, t * ids_stride + k);
        key[k] = e < 0 ? INT32_MAX : e;
        idx[k] = k;
    }
    for (int a = 1; a < top_k; ++a) {
        int kv = key[a], iv = idx[a], b = a - 1;
        while (b >= 0 && key[b] > kv) {
            key[b + 1] = key[b];
            idx[b + 1] = idx[b];
            --b;
        }
        key[b + 1] = kv;
        idx[b + 1] = iv;
    }
    // the slots' contribution rows in summation order: their own positions, or where `rows` says
    // they landed (-1: none)
    int64_t row[kMaxTopK];
    for (int k = 0; k < top_k; ++k)
        row[k] = key[k] == INT32_MAX ? -1 : (rows ? rows[t * top_k + idx[k]] : t * top_k + idx[k]);
    constexpr int kBatch = 8;   // contributions loaded together, then added in order
    for (int64_t c = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; c < hidden;
         c += int64_t(gridDim.x) * blockDim.x) {
        float acc = 0.f;
        for (int k0 = 0; k0 < top_k; k0 += kBatch) {
            float v[kBatch];
#pragma unroll
            for (int j = 0; j < kBatch; ++j) {
                const int64_t r = k0 + j < top_k ? row[k0 + j] : -1;
                v[j] = r >= 0 ? __ldcg(contrib + r * hidden + c) : 0.f;
            }
#pragma unroll
            for (int j = 0; j < kBatch; ++j)
                if (k0 + j < top_k && row[k0 + j] >= 0) acc += v[j];
        }
        out[t * out_stride + c] = acc;
    }
}

}  // namespace

size_t plan_smem_bytes(int n_experts) {
    return sizeof(int) * size_t(kPlanWarps) * size_t(n_experts);
}

int plan_validate(int64_t n_tokens, int top_k, int n_experts) {
    if (n_tokens < 0 || top_k <= 0) return fail(VY_ERR_INVALID, "n_tokens %lld top_k %d", (long long)n_tokens, top_k);
    if (top_k > kMaxTopK) return fail(VY_ERR_UNSUPPORTED, "top_k %d > %d", top_k, kMaxTopK);
    if (n_experts <= 0 || n_experts > kMaxExperts)
        return fail(VY_ERR_UNSUPPORTED, "n_experts %d (1..%d supported)", n_experts, kMaxExperts);
    if (n_tokens * top_k > int64_t(kPlanWarps) * 65535)
        return fail(VY_ERR_UNSUPPORTED, "%lld routed rows in one call (max %d)",
                    (long long)(n_tokens * top_k), kPlanWarps * 65535);
    return VY_OK;
}

int launch_plan(const PlanArgs& p, int sm_count, cudaStream_t stream) {
    size_t smem = plan_smem_bytes(p.n_experts);
    const int st = once_per_device(
        reinterpret_cast<const void*>(plan_kernel),
        [](int, void*) -> int {
            const cudaError_t e = cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                       static_cast<int>(plan_smem_bytes(kMaxExperts)));
            return e == cudaSuccess ? VY_OK : fail(VY_ERR_CUDA, "routing plan shared memory: %s", cudaGetErrorString(e));
        },
        nullptr);
    if (st != VY_OK) return st;
    // a decode-sized plan sorts with as many threads as the next power of two of its rows (the
    // fewer warps, the cheaper every block barrier); the counting sort takes the full block
    const int64_t n = p.n_tokens * p.top_k;
    int threads = kPlanThreads;
    if (n <= kSmallPlan) {
        threads = 64;
        while (threads < n) threads <<= 1;
    }
    int perm_blocks = 0;
    if (p.x_perm) {
        int64_t groups = p.n_tokens * (p.hidden / 8);
        int64_t b = (groups + threads - 1) / threads;
        perm_blocks = static_cast<int>(b < 4 * sm_count ? b : 4 * sm_count);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(1 + perm_blocks));
    cfg.blockDim = dim3(static_cast<unsigned>(threads));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, plan_kernel, p);
    if (e != cudaSuccess) return fail(VY_ERR_CUDA, "routing plan launch: %s", cudaGetErrorString(e));
    return check_launch("routing plan");
}

// out[t] = token t's contributions in the plan's slot order (ascending expert id, then slot;
// dropped rows are -1 and add nothing), fp32.
__global__ void __launch_bounds__(256) slot_combine_kernel(const float* __restrict__ contrib,
                                                           const int32_t* __restrict__ slot_order,
                                                           int64_t n_tokens, int top_k, int hidden,
                                                           float* out, int64_t out_stride) {
    constexpr int kBatch = 8;   // slots whose row ids, then contributions, are loaded together
    grid_dependency_wait();
    grid_dependents_launch();   // the next call's plan may be scheduled; it waits for this grid
    for (int64_t t = blockIdx.y; t < n_tokens; t += gridDim.y)
    for (int c = (blockIdx.x * blockDim.x + threadIdx.x) * 4; c < hidden; c += gridDim.x * blockDim.x * 4) {
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int k0 = 0; k0 < top_k; k0 += kBatch) {
            int row[kBatch];
            float4 v[kBatch];
#pragma unroll
            for (int j = 0; j < kBatch; ++j) row[j] = k0 + j < top_k ? __ldg(slot_order + t * top_k + k0 + j) : -1;
#pragma unroll
            for (int j = 0; j < kBatch; ++j)
                if (row[j] >= 0) v[j] = __ldcg(reinterpret_cast<const float4*>(contrib + int64_t(row[j]) * hidden + c));
            // ascending expert id, then slot: the order the rows were filed in
#pragma unroll
            for (int j = 0; j < kBatch; ++j) {
                if (row[j] < 0) continue;
                a.x += v[j].x;
                a.y += v[j].y;
                a.z += v[j].z;
                a.w += v[j].w;
            }
        }
        float* o = out + t * out_stride + c;
        o[0] = a.x;
        o[1] = a.y;
        o[2] = a.z;
        o[3] = a.w;
    }
}

int launch_slot_combine(const float* contrib, const int32_t* slot_order, int64_t n_tokens, int top_k, int hidden,
                        float* out, int64_t out_stride, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((hidden / 4 + 255) / 256),
                       static_cast<unsigned>(n_tokens < 65535 ? n_tokens : 65535));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, slot_combine_kernel, contrib, slot_order, n_tokens, top_k, hidden,
                                       out, out_stride);
    if (e != cudaSuccess) return fail(VY_ERR_CUDA, "combine launch: %s", cudaGetErrorString(e));
    return VY_OK;
}

// The same sum over a token's routed slots, then the model's epilogue with its shared expert in
// slot top_k - 1: result[t] = act(act(routed sum) + act(shared c))
// (vaayu/packed_expert_kernels.py:502-508).  `out`, when given, receives the routed fp32 sum.
template <int ACT>
__global__ void __launch_bounds__(256) shared_combine_kernel(const float* __restrict__ contrib,
                                                             const int32_t* __restrict__ slot_order,
                                                             int64_t n_tokens, int top_k, int hidden,
                                                             float* out, int64_t out_stride,
                                                             uint16_t* result, int64_t result_stride) {
    constexpr int kBatch = 8;
    grid_dependency_wait();
    grid_dependents_launch();
    for (int64_t t = blockIdx.y; t < n_tokens; t += gridDim.y)
    for (int c = (blockIdx.x * blockDim.x + threadIdx.x) * 4; c < hidden; c += gridDim.x * blockDim.x * 4) {
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f), sh = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int k0 = 0; k0 < top_k; k0 += kBatch) {
            int row[kBatch];
            float4 v[kBatch];
#pragma unroll
            for (int j = 0; j < kBatch; ++j) row[j] = k0 + j < top_k ? __ldg(slot_order + t * top_k + k0 + j) : -1;
#pragma unroll
            for (int j = 0; j < kBatch; ++j)
                if (row[j] >= 0) v[j] = __ldcg(reinterpret_cast<const float4*>(contrib + int64_t(row[j]) * hidden + c));
#pragma unroll
            for (int j = 0; j < kBatch; ++j) {
                if (row[j] < 0) continue;
                if (row[j] % top_k == top_k - 1) {   // the shared expert's slot
                    sh = v[j];
                    continue;
                }
                a.x += v[j].x;
                a.y += v[j].y;
                a.z += v[j].z;
                a.w += v[j].w;
            }
        }
        if (out) {
            float* o = out + t * out_stride + c;
            o[0] = a.x;
            o[1] = a.y;
            o[2] = a.z;
            o[3] = a.w;
        }
        const float ra[4] = {a.x, a.y, a.z, a.w}, rs[4] = {sh.x, sh.y, sh.z, sh.w};
        uint16_t* r = result + t * result_stride + c;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            r[i] = static_cast<uint16_t>(act_bits<ACT>(round_act<ACT>(ra[i]) + round_act<ACT>(rs[i])));
    }
}

int launch_shared_combine(const float* contrib, const int32_t* slot_order, int64_t n_tokens, int top_k, int hidden,
                          float* out, int64_t out_stride, void* result, int64_t result_stride, int act,
                          cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((hidden / 4 + 255) / 256),
                       static_cast<unsigned>(n_tokens < 65535 ? n_tokens : 65535));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    uint16_t* res = static_cast<uint16_t*>(result);
    cudaError_t e = act == VY_BF16
        ? cudaLaunchKernelEx(&cfg, shared_combine_kernel<VY_BF16>, contrib, slot_order, n_tokens, top_k, hidden,
                             out, out_stride, res, result_stride)
        : cudaLaunchKernelEx(&cfg, shared_combine_kernel<VY_F16>, contrib, slot_order, n_tokens, top_k, hidden,
                             out, out_stride, res, result_stride);
    if (e != cudaSuccess) return fail(VY_ERR_CUDA, "shared-expert combine launch: %s", cudaGetErrorString(e));
    return VY_OK;
}

// The layer's final combine: the routed fp32 sum into `out`, or with shared_last the epilogue
// with the shared expert into `result` as well.
int launch_layer_combine(const vy_moe_call* c, const float* contrib, const int32_t* slot_order, cudaStream_t s) {
    const int hidden = c->geom->hidden;
    if (c->shared_last)
        return launch_shared_combine(contrib, slot_order, c->n_tokens, c->top_k, hidden, c->out, c->out_row_stride,
                                     c->result, c->result_row_stride, c->act_dtype, s);
    return launch_slot_combine(contrib, slot_order, c->n_tokens, c->top_k, hidden, c->out, c->out_row_stride, s);
}

int launch_combine(const float* contrib, const void* ids, bool ids64, int64_t n_tokens,
                   int top_k, int64_t hidden, float* out, int64_t out_stride, int sm_count,
                   cudaStream_t stream, const int64_t* rows, int64_t ids_stride, bool chained) {
    if (n_tokens == 0) return VY_OK;
    int bx = static_cast<int>((hidden + 255) / 256);
    if (bx > 8) bx = 8;
    (void)sm_count;
    dim3 grid(bx, static_cast<unsigned>(n_tokens));
    const int64_t stride = ids_stride > 0 ? ids_stride : top_k;
    if (chained) {
        const cudaError_t e = launch_chained(combine_kernel, grid, dim3(256), 0, stream, contrib, ids, ids64, stride,
                                             n_tokens, top_k, hidden, out, out_stride, rows);
        if (e != cudaSuccess) return fail(VY_ERR_CUDA, "combine launch: %s", cudaGetErrorString(e));
    } else {
        combine_kernel<<<grid, 256, 0, stream>>>(contrib, ids, ids64, stride, n_tokens, top_k, hidden, out,
                                                 out_stride, rows);
    }
    return check_launch("combine");
}

// out[i] = parts[0][i] + parts[1][i] + ... in part order, one fp32 add each (float4 lanes).
__global__ void __launch_bounds__(256) sum_ordered_kernel(const float4* __restrict__ parts, int n_parts, int64_t n4,
                                                          float4* out) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n4; i += int64_t(gridDim.x) * blockDim.x) {
        float4 a = parts[i];
        for (int q = 1; q < n_parts; ++q) {
            const float4 v = parts[int64_t(q) * n4 + i];
            a.x += v.x;
            a.y += v.y;
            a.z += v.z;
            a.w += v.w;
        }
        out[i] = a;
    }
}

}  // namespace vy

using namespace vy;

extern "C" int vy_sum_ordered(const float* parts, int32_t n_parts, int64_t n, float* out, void* stream) {
    int st;
    const DeviceInfo* dev = device_info(&st);
    if (!dev) return st;
    if (n_parts < 1 || n < 0) return fail(VY_ERR_INVALID, "%d parts of %lld", n_parts, (long long)n);
    if (n == 0) return ok();
    if (!parts || !out) return fail(VY_ERR_INVALID, "null pointer");
    if (n % 4 || !aligned16(parts) || !aligned16(out))
        return fail(VY_ERR_ALIGNMENT, "parts / out must be 16-byte aligned with n a multiple of 4");
    const int64_t n4 = n / 4;
    int64_t blocks = (n4 + 255) / 256;
    if (blocks > 8 * dev->sm_count) blocks = 8 * dev->sm_count;
    sum_ordered_kernel<<<static_cast<unsigned>(blocks), 256, 0, as_stream(stream)>>>(
        reinterpret_cast<const float4*>(parts), n_parts, n4, reinterpret_cast<float4*>(out));
    return check_launch("vy_sum_ordered");
}

extern "C" int vy_moe_route_permute(const void* ids, int32_t ids_dtype, int64_t n_tokens,
                                    int32_t top_k, int32_t n_experts, int32_t* order,
                                    int32_t* live_expert, int32_t* live_start,
                                    int32_t* slot_order, int32_t* counters, void* stream) {
    int st;
    const DeviceInfo* dev = device_info(&st);
    if (!dev) return st;
    if ((st = plan_validate(n_tokens, top_k, n_experts)) != VY_OK) return st;
    if (ids_dtype != VY_I32 && ids_dtype != VY_I64) return fail(VY_ERR_UNSUPPORTED, "id dtype %d", ids_dtype);
    if (!order || !live_expert || !live_start || !slot_order || !counters)
        return fail(VY_ERR_INVALID, "null output");
    if (n_tokens > 0 && !ids) return fail(VY_ERR_INVALID, "null ids");
    PlanArgs p{};
    p.ids = ids;
    p.ids64 = ids_dtype == VY_I64;
    p.ids_stride = top_k;
    p.id_base = 0;
    p.n_tokens = n_tokens;
    p.top_k = top_k;
    p.n_experts = n_experts;
    p.order = order;
    p.live_expert = live_expert;
    p.live_start = live_start;
    p.slot_order = slot_order;
    p.counters = counters;
    p.unit_start = nullptr;
    p.tok_per_unit = 0;
    return launch_plan(p, dev->sm_count, as_stream(stream));
}

extern "C" int vy_moe_topk_softmax(const void* logits, int32_t logit_dtype, int64_t row_stride,
                                   int64_t n_tokens, int32_t n_experts, int32_t top_k,
                                   float* weights, int64_t* ids, void* stream) {
    int st;
    const DeviceInfo* dev = device_info(&st);
    if (!dev) return st;
    if (n_tokens < 0 || n_experts <= 0 || top_k <= 0 || top_k > n_experts)
        return fail(VY_ERR_INVALID, "n_tokens %lld n_experts %d top_k %d", (long long)n_tokens, n_experts, top_k);
    if (top_k > kMaxTopK) return fail(VY_ERR_UNSUPPORTED, "top_k %d > %d", top_k, kMaxTopK);
    if (n_tokens == 0) return ok();
    if (!logits || !weights || !ids) return fail(VY_ERR_INVALID, "null pointer");
    const int warps = 8;
    const unsigned grid = static_cast<unsigned>((n_tokens + warps - 1) / warps);
    cudaStream_t s = as_stream(stream);
    switch (logit_dtype) {
        case VY_F32: topk_softmax_kernel<VY_F32><<<grid, warps * 32, 0, s>>>(logits, row_stride, n_tokens, n_experts, top_k, weights, ids); break;
        case VY_BF16: topk_softmax_kernel<VY_BF16><<<grid, warps * 32, 0, s>>>(logits, row_stride, n_tokens, n_experts, top_k, weights, ids); break;
        case VY_F16: topk_softmax_kernel<VY_F16><<<grid, warps * 32, 0, s>>>(logits, row_stride, n_tokens, n_experts, top_k, weights, ids); break;
        default: return fail(VY_ERR_UNSUPPORTED, "logit dtype %d", logit_dtype);
    }
    return check_launch("vy_moe_topk_softmax");
}

extern "C" int vy_moe_combine(const float* contrib, const void* expert_ids, int32_t ids_dtype,
                              int64_t n_tokens, int32_t top_k, int64_t hidden, float* out,
                              int64_t out_row_stride, void* stream) {
    int st;
    const DeviceInfo* dev = device_info(&st);
    if (!dev) return st;
    if (n_tokens < 0 || top_k <= 0 || hidden < 0) return fail(VY_ERR_INVALID, "bad sizes");
    if (top_k > kMaxTopK) return fail(VY_ERR_UNSUPPORTED, "top_k %d > %d", top_k, kMaxTopK);
    if (ids_dtype != VY_I32 && ids_dtype != VY_I64) return fail(VY_ERR_UNSUPPORTED, "id dtype %d", ids_dtype);
    if (n_tokens == 0 || hidden == 0) return ok();
    if (!contrib || !expert_ids || !out) return fail(VY_ERR_INVALID, "null pointer");
    return launch_combine(contrib, expert_ids, ids_dtype == VY_I64, n_tokens, top_k, hidden, out,
                          out_row_stride, dev->sm_count, as_stream(stream));
}
