// vy_ep.cu -- the expert-parallel exchange around the expert kernels: the dispatch plan that
// addresses every (token, slot) row of a rank's batch to the rank holding its expert and packs
// the send buffers of fixed-capacity, equal-split all-to-alls, and the combine that reads the
// returned contributions through the same slot map.
//
// The exchange itself is NCCL's (torch.distributed over NVLink): these kernels only prepare and
// consume this GPU's own buffers, so no kernel here reads another GPU's memory.
//
//   ep_plan_kernel   one CTA: per-warp counts of the rows bound for each destination over
//                    contiguous row segments, a prefix over the warps (warp order = row order),
//                    then each row's position among its destination's rows (stable), its slot,
//                    local expert id and fp32 routing weight.
//   ep_pack_kernel   grid-wide: a warp per row copies the token's activations into its slot
//                    (16-byte vectors when aligned); every slot past its destination's count gets
//                    expert id -1, which the receiving rank's routing plan drops.
#include "vy_moe.cuh"

namespace vy {
namespace {

constexpr int kEpThreads = 1024;
constexpr int kEpWarps = kEpThreads / 32;
constexpr int kMaxRanks = 64;

struct EpPlanArgs {
    const void* ids;
    bool ids64;
    int64_t ids_stride;        // elements between tokens' id rows
    int64_t n_tokens;
    int top_k;
    int n_ranks, per_rank;
    bool interleaved;          // expert e on rank e % n_ranks (else e / per_rank)
    const void* w;
    int w_dtype;
    int64_t w_tok_stride, w_slot_stride;
    int64_t capacity;          // slots per destination
    int32_t* send_ids;
    float* send_w;
    int64_t* slot_of_row;
    int32_t* counts;
    int32_t* wanted;           // optional: rows bound for each destination before the capacity cut
};

// Destination rank of row j = t * top_k + k (-1: an id outside the experts), and its local id.
__device__ __forceinline__ int ep_dest(const EpPlanArgs& p, int64_t j, int* local) {
    const int64_t t = j / p.top_k, k = j - t * p.top_k;
    int64_t e;
    if (p.ids64) {
        e = reinterpret_cast<const int64_t*>(p.ids)[t * p.ids_stride + k];
    } else {
        e = reinterpret_cast<const int32_t*>(p.ids)[t * p.ids_stride + k];
    }
    if (e < 0 || e >= int64_t(p.n_ranks) * p.per_rank) return -1;
    const int ei = static_cast<int>(e);
    int d;
    if (p.interleaved) {
        d = ei % p.n_ranks;
        *local = ei / p.n_ranks;
    } else {
        d = ei / p.per_rank;
        *local = ei - d * p.per_rank;
    }
    return d;
}

__global__ void __launch_bounds__(kEpThreads) ep_plan_kernel(EpPlanArgs p) {
    __shared__ int run[kEpWarps][kMaxRanks];   // per warp and destination: count, then next position
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t n = p.n_tokens * p.top_k;
    const int64_t seg = (n + kEpWarps - 1) / kEpWarps;
    const int64_t lo = warp * seg, hi = lo + seg < n ? lo + seg : n;
    for (int d = lane; d < p.n_ranks; d += 32) run[warp][d] = 0;
    __syncwarp();
    // 1. each warp counts its segment's rows per destination
    for (int64_t base = lo; base < hi; base += 32) {
        const int64_t row = base + lane;
        int local = 0;
        const int d = row < hi ? ep_dest(p, row, &local) : -1;
        const unsigned same = __match_any_sync(0xffffffffu, d);
        if (d >= 0 && lane == __ffs(same) - 1) run[warp][d] += __popc(same);
        __syncwarp();
    }
    __syncthreads();
    // 2. per destination, warp by warp: each warp's first position among the destination's rows
    if (threadIdx.x < p.n_ranks) {
        const int d = threadIdx.x;
        int total = 0;
        for (int w = 0; w < kEpWarps; ++w) {
            const int c = run[w][d];
            run[w][d] = total;
            total += c;
        }
        p.counts[d] = total < p.capacity ? total : static_cast<int>(p.capacity);
        if (p.wanted) p.wanted[d] = total;
    }
    __syncthreads();
    // 3. each row's slot: its warp's next position for the destination + its rank among the
    //    lanes with the same destination (rows past the capacity are dropped: slot -1)
    for (int64_t base = lo; base < hi; base += 32) {
        const int64_t row = base + lane;
        int local = 0;
        const int d = row < hi ? ep_dest(p, row, &local) : -1;
        const unsigned same = __match_any_sync(0xffffffffu, d);
        int64_t slot = -1;
        if (d >= 0) {
            const int64_t pos = run[warp][d] + __popc(same & ((1u << lane) - 1u));
            if (pos < p.capacity) {
                slot = d * p.capacity + pos;
                const int64_t t = row / p.top_k, k = row - t * p.top_k;
                p.send_ids[slot] = local;
                p.send_w[slot] = load_as_float(p.w, p.w_dtype, t * p.w_tok_stride + k * p.w_slot_stride);
            }
        }
        if (row < hi) p.slot_of_row[row] = slot;
        __syncwarp();   // every lane has read its warp's position before the leaders move it on
        if (d >= 0 && lane == __ffs(same) - 1) run[warp][d] += __popc(same);
        __syncwarp();
    }
}

struct EpPackArgs {
    const uint16_t* x;
    int64_t x_stride;          // elements between token rows
    int64_t hidden;
    int top_k;
    int64_t n_rows;
    const int64_t* slot_of_row;
    uint16_t* send_x;
    bool vec;                  // 16-byte copies (x, its stride, hidden and send_x all allow them)
    int64_t n_slots, capacity;
    const int32_t* counts;
    int32_t* send_ids;
};

__global__ void __launch_bounds__(256) ep_pack_kernel(EpPackArgs p) {
    const int lane = threadIdx.x & 31;
    const int64_t gw = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5;
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t row = gw; row < p.n_rows; row += nwarps) {
        const int64_t slot = p.slot_of_row[row];
        if (slot < 0) continue;
        const uint16_t* src = p.x + (row / p.top_k) * p.x_stride;
        uint16_t* dst = p.send_x + slot * p.hidden;
        if (p.vec) {
            const int64_t n16 = p.hidden / 8;
            for (int64_t i = lane; i < n16; i += 32)
                reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
        } else {
            for (int64_t i = lane; i < p.hidden; i += 32) dst[i] = src[i];
        }
    }
    for (int64_t s = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; s < p.n_slots;
         s += int64_t(gridDim.x) * blockDim.x) {
        const int64_t d = s / p.capacity;
        if (s - d * p.capacity >= p.counts[d]) p.send_ids[s] = -1;
    }
}

}  // namespace
}  // namespace vy

using namespace vy;

extern "C" int vy_ep_dispatch_plan(const void* ids, int32_t ids_dtype, int64_t ids_row_stride, int64_t n_tokens,
                                   int32_t top_k, int32_t n_ranks, int32_t experts_per_rank, int32_t placement,
                                   const void* weights, int32_t w_dtype, int64_t w_tok_stride,
                                   int64_t w_slot_stride, const void* x, int32_t x_dtype, int64_t x_row_stride,
                                   int64_t hidden, int64_t capacity, int32_t* send_ids, float* send_w,
                                   void* send_x, int64_t* slot_of_row, int32_t* counts, int32_t* wanted,
                                   void* stream) {
    int st;
    const DeviceInfo* dev = device_info(&st);
    if (!dev) return st;
    if (n_tokens < 0 || top_k <= 0 || hidden <= 0 || capacity < 0)
        return fail(VY_ERR_INVALID, "n_tokens %lld top_k %d hidden %lld capacity %lld", (long long)n_tokens,
                    top_k, (long long)hidden, (long long)capacity);
    if (n_ranks < 1 || n_ranks > kMaxRanks || experts_per_rank < 1)
        return fail(VY_ERR_UNSUPPORTED, "%d ranks of %d experts (1..%d ranks)", n_ranks, experts_per_rank,
                    kMaxRanks);
    if (int64_t(n_ranks) * experts_per_rank > INT32_MAX || int64_t(n_ranks) * capacity > INT32_MAX ||
        n_tokens * top_k > INT32_MAX)
        return fail(VY_ERR_UNSUPPORTED, "sizes beyond 32-bit slot and expert indices");
    if (placement != 0 && placement != 1)
        return fail(VY_ERR_INVALID, "placement %d (0 contiguous, 1 interleaved)", placement);
    if (ids_dtype != VY_I32 && ids_dtype != VY_I64) return fail(VY_ERR_UNSUPPORTED, "id dtype %d", ids_dtype);
    if (w_dtype != VY_BF16 && w_dtype != VY_F16 && w_dtype != VY_F32)
        return fail(VY_ERR_UNSUPPORTED, "routing-weight dtype %d", w_dtype);
    if (x_dtype != VY_BF16 && x_dtype != VY_F16) return fail(VY_ERR_UNSUPPORTED, "activation dtype %d", x_dtype);
    if (ids_row_stride < top_k || x_row_stride < hidden)
        return fail(VY_ERR_INVALID, "ids row stride %lld / x row stride %lld", (long long)ids_row_stride,
                    (long long)x_row_stride);
    if (!send_ids || !send_w || !send_x || !counts || (n_tokens > 0 && (!ids || !weights || !x || !slot_of_row)))
        return fail(VY_ERR_INVALID, "null pointer");
    cudaStream_t s = as_stream(stream);
    EpPlanArgs p{};
    p.ids = ids;
    p.ids64 = ids_dtype == VY_I64;
    p.ids_stride = ids_row_stride;
    p.n_tokens = n_tokens;
    p.top_k = top_k;
    p.n_ranks = n_ranks;
    p.per_rank = experts_per_rank;
    p.interleaved = placement == 1;
    p.w = weights;
    p.w_dtype = w_dtype;
    p.w_tok_stride = w_tok_stride;
    p.w_slot_stride = w_slot_stride;
    p.capacity = capacity;
    p.send_ids = send_ids;
    p.send_w = send_w;
    p.slot_of_row = slot_of_row;
    p.counts = counts;
    p.wanted = wanted;
    ep_plan_kernel<<<1, kEpThreads, 0, s>>>(p);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(VY_ERR_CUDA, "dispatch plan launch: %s", cudaGetErrorString(e));

    EpPackArgs q{};
    q.x = static_cast<const uint16_t*>(x);
    q.x_stride = x_row_stride;
    q.hidden = hidden;
    q.top_k = top_k;
    q.n_rows = n_tokens * top_k;
    q.slot_of_row = slot_of_row;
    q.send_x = static_cast<uint16_t*>(send_x);
    q.vec = aligned16(x) && aligned16(send_x) && x_row_stride % 8 == 0 && hidden % 8 == 0;
    q.n_slots = int64_t(n_ranks) * capacity;
    q.capacity = capacity;
    q.counts = counts;
    q.send_ids = send_ids;
    const int64_t work = q.n_rows > q.n_slots / 32 ? q.n_rows : q.n_slots / 32;   // warps' worth of work
    int64_t blocks = (work + 7) / 8;
    if (blocks > 8 * dev->sm_count) blocks = 8 * dev->sm_count;
    if (blocks < 1) blocks = 1;
    if (q.n_slots > 0 || q.n_rows > 0) ep_pack_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(q);
    return check_launch("vy_ep_dispatch_plan");
}

extern "C" int vy_ep_combine(const float* back, const int64_t* slot_of_row, const void* expert_ids,
                             int32_t ids_dtype, int64_t ids_row_stride, int64_t n_tokens, int32_t top_k,
                             int64_t hidden, float* out, int64_t out_row_stride, void* stream) {
    int st;
    const DeviceInfo* dev = device_info(&st);
    if (!dev) return st;
    if (n_tokens < 0 || top_k <= 0 || hidden < 0) return fail(VY_ERR_INVALID, "bad sizes");
    if (n_tokens > 65535)
        return fail(VY_ERR_UNSUPPORTED, "%lld tokens in one combine (max 65535)", (long long)n_tokens);
    if (top_k > kMaxTopK) return fail(VY_ERR_UNSUPPORTED, "top_k %d > %d", top_k, kMaxTopK);
    if (ids_dtype != VY_I32 && ids_dtype != VY_I64) return fail(VY_ERR_UNSUPPORTED, "id dtype %d", ids_dtype);
    if (out_row_stride < hidden) return fail(VY_ERR_INVALID, "out row stride %lld", (long long)out_row_stride);
    if (ids_row_stride != 0 && ids_row_stride < top_k)
        return fail(VY_ERR_INVALID, "ids row stride %lld < top_k %d", (long long)ids_row_stride, top_k);
    if (n_tokens == 0 || hidden == 0) return ok();
    if (!back || !slot_of_row || !expert_ids || !out) return fail(VY_ERR_INVALID, "null pointer");
    return launch_combine(back, expert_ids, ids_dtype == VY_I64, n_tokens, top_k, hidden, out, out_row_stride,
                          dev->sm_count, as_stream(stream), slot_of_row, ids_row_stride);
}
