// vy_prefill.cu -- the prefill expert layer as tcgen05 grouped GEMMs (accumulators in TMEM).
//
//   plan (vy_route.cu)   rows grouped by expert; the pass table holds one entry per 128-row unit
//                        of a live expert (stream pointers, first sorted row, row count)
//   gather_kernel        x rows in sorted order -> x_sorted, 8-element groups permuted the way the
//                        dequantised pairs come out (code j pairs with code j + 4), so A and B
//                        share one consistent K order
//   gemm_kernel<0>       h = act(act(silu(act(x Wg^T))) * act(x Wu^T)), 128 rows x 128 columns
//                        (128 gate + 128 up weight rows per CTA)
//   gemm_kernel<1>       c = act(h Wd^T) * w (one fp32 rounding), 128 rows x 256 columns,
//                        scattered to the row ids
//   slot_combine_kernel  each token's contributions in ascending expert id, then slot
//
// A GEMM CTA: 8 dequant warps, 16 fold warps, one control warp group (one thread of it works);
// `setmaxnreg` gives the fold warps the registers the other roles do not need.
//   dequant  one thread per row of the 256-row weight tile (64 codes per stage): it copies the
//            row's packed codes into a private cp.async ring (the row's scale and zero words
//            stream through registers, a word ahead), dequantises them with the reference's exact
//            rounding of every weight (sub.rn then mul.rn on activation-dtype pairs) and stores
//            16-byte chunks into the weight tile in the 128-byte-swizzled K-major layout the
//            tensor core reads; each warp then arrives once on the stage's barrier.
//   control  one thread issues tcgen05.mma M=128 N=256 K=16 (and nothing else: the tensor core
//            queues only a few MMAs, so other work in that thread lets it drain); a second thread
//            loads the 128-row activation tiles with one TMA box each (same swizzle, no multicast).
//   fold     K is cut into chunks of kChunk stages.  Each chunk accumulates from zero in one of
//            two TMEM buffers (2 x 256 columns); the fold warps read it with tcgen05.ld and add it
//            into fp32 sums held in their registers with round-to-nearest adds (paired fp32 adds),
//            while the tensor core fills the other buffer.  The tensor core's own accumulate
//            truncates against the accumulator's magnitude, so one chain over the whole K drifts
//            (biased) from the fp32 sum; short chunks keep every output as close to the correctly
//            rounded dot product as the decode path's.  The fold warps then run the epilogue from
//            their registers.
// Every barrier wait is bounded: on a timeout the CTA records an error flag, drains what it
// issued, frees TMEM and returns.
#include <cuda.h>

#include <mutex>

#include "vy_moe.cuh"

namespace vy {
namespace {

constexpr int kBM = 128, kBK = 64;    // one MMA: 128 rows, K = 64 per stage
constexpr int kUnit = kBM;            // activation rows per CTA
constexpr int kBN = 256;              // a CTA's N: 128 gate + 128 up rows, or 256 down rows
constexpr int kGuCols = kBN / 2;      // intermediate columns of one gate/up CTA
#ifndef VY_PF_ASTAGES
#define VY_PF_ASTAGES 6
#endif
#ifndef VY_PF_BSTAGES
#define VY_PF_BSTAGES 3
#endif
#ifndef VY_PF_PACK
#define VY_PF_PACK 4
#endif
#ifndef VY_PF_CHUNK
#define VY_PF_CHUNK 4
#endif
constexpr int kAStages = VY_PF_ASTAGES;   // activation-tile ring (TMA)
constexpr int kBStages = VY_PF_BSTAGES;   // weight-tile ring (dequant warps)
constexpr int kPack = VY_PF_PACK;         // packed-code staging depth, private to each dequant thread
constexpr int kChunk = VY_PF_CHUNK;       // stages one TMEM accumulation runs before it is folded
constexpr int kDqWarps = 8;           // one dequant thread per weight-tile row
constexpr int kDqThreads = kDqWarps * 32;
constexpr int kFoldWarps = 16;        // 4 lane quarters x 4 column quarters
constexpr int kCtlWarp = kDqWarps + kFoldWarps;   // first warp of the control warp group
constexpr int kThreads = (kCtlWarp + 4) * 32;     // 28 warps: 7 warp groups
// Registers per thread after `setmaxnreg` (warp-group granular).  The launch gives every thread
// the same count; the kernel only runs when that launch budget covers this split (host check).
constexpr int kDqRegs = 56, kFoldRegs = 88, kCtlRegs = 40;
constexpr int kRegSplit = (kDqWarps * kDqRegs + kFoldWarps * kFoldRegs + 4 * kCtlRegs) * 32;
static_assert(kDqWarps % 4 == 0 && kFoldWarps % 4 == 0 && kCtlWarp % 4 == 0, "roles are whole warp groups");
static_assert(kDqThreads == kBN, "one dequant thread per weight-tile row");
constexpr uint32_t kBufCols = kBN;            // one accumulator buffer: 128 lanes x N = 256
constexpr uint32_t kTmemCols = 2 * kBufCols;  // double-buffered: 512 columns
constexpr int kFoldVals = kBN / 4;            // fp32 sums one fold thread holds (its row, 64 columns)
constexpr uint64_t kWaitNs = 2000000000ull;   // a barrier wait gives up after 2 s
constexpr int kTileBytes = kUnit * kBK * 2;   // 16 KB: one 128 x 64 activation tile

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ── mbarrier / TMA / tcgen05 wrappers ───────────────────────────────────────────────────────

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// The same test, but a thread whose phase is not complete yet may be suspended (woken when it
// completes) for up to `hint_ns` instead of returning at once: waiting warps then take no issue
// slots from the working ones.
__device__ __forceinline__ bool mbar_try_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}
constexpr uint32_t kSuspendNs = 100000;   // a waiting thread rechecks abort / timeout every 0.1 ms
__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait (try_wait suspends in hardware between polls); false once the CTA has aborted, or
// after `limit_ns`, when it aborts the CTA itself (error bit 4).
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                              int32_t* err, uint64_t limit_ns) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = now_ns();
    for (;;) {
        if (mbar_try_sleep(bar, parity, kSuspendNs)) return true;
        if (*abort_flag) return false;
        if (now_ns() - t0 > limit_ns) {
            *abort_flag = 1;
            atomicOr(err, 4);
            return false;
        }
    }
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int32_t* err) {
    return mbar_wait_for(bar, parity, abort_flag, err, kWaitNs);
}

// Bounded wait that ignores the abort flag: drains work already issued (TMA loads, MMAs) before
// the CTA releases its shared memory and TMEM (error bit 8 if even that times out).
__device__ __forceinline__ bool mbar_drain(uint64_t* bar, uint32_t parity, int32_t* err) {
    const uint64_t t0 = now_ns();
    for (;;) {
        if (mbar_try_sleep(bar, parity, kSuspendNs)) return true;
        if (now_ns() - t0 > kWaitNs) {
            atomicOr(err, 8);
            return false;
        }
    }
}

__device__ __forceinline__ uint2 ld_nc_v2(const void* p) {
    uint2 v;
    asm volatile("ld.global.nc.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

// One row's scale (or zero-point) elements [first, last] read as the aligned 8-byte words that
// hold them (2^LG elements per word): the word of the current stage sits in a register and the
// next one is loaded when the current one is entered, a whole word period before it is needed.
// Only words holding an element of the row are read.
template <int LG>
struct WordStream {
    const uint2* words;
    uint32_t last;      // the row's last element
    uint32_t wi;        // index of the word in `cur`
    uint2 cur, nxt;
    __device__ __forceinline__ void start(const void* base, uint32_t first_elem, uint32_t last_elem, bool go) {
        words = reinterpret_cast<const uint2*>(base);
        last = last_elem;
        wi = first_elem >> LG;
        cur = go ? ld_nc_v2(words + wi) : make_uint2(0u, 0u);
        nxt = (go && ((wi + 1) << LG) <= last) ? ld_nc_v2(words + wi + 1) : make_uint2(0u, 0u);
    }
    // the word holding element e (e never moves more than one word per call)
    __device__ __forceinline__ uint2 at(uint32_t e, bool go) {
        const uint32_t w = e >> LG;
        if (w != wi) {
            wi = w;
            cur = nxt;
            if (go && ((w + 1) << LG) <= last) nxt = ld_nc_v2(words + w + 1);
        }
        return cur;
    }
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void umma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// Two fp32 round-to-nearest adds in one instruction (each half of the pair rounds on its own,
// exactly as two separate adds do).
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t pack_f32x2(uint32_t lo, uint32_t hi) {
    uint64_t d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(lo), "r"(hi));
    return d;
}
__device__ __forceinline__ float2 unpack_f32x2(uint64_t v) {
    uint32_t lo, hi;
    asm("mov.b64 {%0, %1}, %2;" : "=r"(lo), "=r"(hi) : "l"(v));
    return make_float2(__uint_as_float(lo), __uint_as_float(hi));
}

// K-major, 128-byte swizzle, 64 bf16 per row, rows 128 bytes apart, 8-row groups 1024 bytes
// apart (SBO); LBO unused for swizzled K-major (1); version 1; layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(const void* tile) {
    const uint64_t addr = smem_u32(tile);
    return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | (uint64_t(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}

// kind::f16 instruction descriptor: fp32 accumulate, A/B bf16 (1) or fp16 (0), both K-major,
// N = kBN, M = kBM.
template <int ACT>
__host__ __device__ constexpr uint32_t idesc_f16() {
    return (1u << 4) | (uint32_t(ACT == VY_BF16 ? 1 : 0) << 7) | (uint32_t(ACT == VY_BF16 ? 1 : 0) << 10) |
           (uint32_t(kBN >> 3) << 17) | (uint32_t(kBM >> 4) << 24);
}

// ── the gather ──────────────────────────────────────────────────────────────────────────────

struct GatherParams {
    const void* x;
    int64_t x_stride;
    int hidden, top_k;
    const int32_t* order;
    const int32_t* live_start;   // live_start[n_live] = rows kept
    const int32_t* counters;
    uint16_t* x_sorted;          // [n, hidden], 8-element groups permuted
};

__global__ void __launch_bounds__(256) gather_kernel(GatherParams p) {
    grid_dependency_wait();
    const int n_rows = p.live_start[p.counters[0]];
    const int groups = p.hidden / 8;
    const int64_t total = int64_t(n_rows) * groups;
    for (int64_t q = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; q < total; q += int64_t(gridDim.x) * blockDim.x) {
        const int pos = static_cast<int>(q / groups), c = static_cast<int>(q - int64_t(pos) * groups) * 8;
        const int row = p.order[pos];
        const uint16_t* src = reinterpret_cast<const uint16_t*>(p.x) + int64_t(row / p.top_k) * p.x_stride + c;
        uint16_t v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = src[j];
        uint4 o;
        o.x = v[0] | (uint32_t(v[4]) << 16);
        o.y = v[1] | (uint32_t(v[5]) << 16);
        o.z = v[2] | (uint32_t(v[6]) << 16);
        o.w = v[3] | (uint32_t(v[7]) << 16);
        *reinterpret_cast<uint4*>(p.x_sorted + int64_t(pos) * p.hidden + c) = o;
    }
}

// ── the GEMM ────────────────────────────────────────────────────────────────────────────────

struct GemmParams {
    int kdim;              // K of this GEMM (hidden for gate/up, inter for down)
    int ndim;              // output features (inter for gate/up, hidden for down)
    int gs_shift;
    int top_k;
    int64_t w_off[2], s_off[2], z_off[2];   // roles: gate, up (KIND 0) or down (KIND 1, [0])
    const PassEntry* passes;
    const int32_t* unit_start;
    int32_t* counters;     // [0] n_live, [2] error flags
    const int32_t* order;
    uint16_t* h_sorted;    // gate/up output [n, inter] (sorted rows, permuted groups)
    uint16_t* h_out;       // optional natural-order h by row id
    float* contrib;        // down output [rows, hidden] by row id
    const void* weights;
    int w_dtype;
    bool w_round;
    int64_t w_tok_stride, w_slot_stride;
    const int32_t* w_index;
};

struct __align__(1024) GemmSmem {
    uint16_t a[kAStages][kUnit * kBK];         // activation tiles (TMA, swizzled): rows 0-127
    uint16_t b[kBStages][kBN * kBK];           // weight tiles: KIND 0 rows 0-127 gate, 128-255 up
    uint4 pack[kPack][2][kDqThreads];          // packed codes (2 chunks of a row), private per thread
    uint64_t full_a[kAStages], full_b[kBStages];
    uint64_t mma_done[kAStages];               // stage s's MMAs complete: barrier s % kAStages
    uint64_t chunk_full[2], chunk_free[2], done;
    uint32_t tmem_base;
    int abort_flag;
};

// The activation-dtype bits of scale element `sub` of an 8-byte scale word.
template <int ACT, int SC>
__device__ __forceinline__ uint32_t scale_bits(uint2 v, int sub) {
    if constexpr (SC == VY_F32) {
        return act_bits<ACT>(__uint_as_float(sub ? v.y : v.x));
    } else {
        const uint32_t w = (sub & 2) ? v.y : v.x;
        const uint32_t b16 = (sub & 1) ? (w >> 16) : (w & 0xFFFFu);
        if constexpr (SC == ACT) {
            return b16;
        } else if constexpr (SC == VY_F16) {
            return act_bits<ACT>(__half2float(__ushort_as_half(static_cast<unsigned short>(b16))));
        } else {
            return act_bits<ACT>(__bfloat162float(__ushort_as_bfloat16(static_cast<unsigned short>(b16))));
        }
    }
}

// KIND 0: 128 gate and the same 128 up rows of the intermediate; the epilogue writes
//         h = act(act(silu(g)) * u).
// KIND 1: 256 rows of down (128 when hidden ends on an odd 128-block); the epilogue writes
//         contributions act(y) * w by row id.
template <int ACT, int SC, bool ZERO, int KIND>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, GemmParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    GemmSmem& S = *reinterpret_cast<GemmSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    grid_dependency_wait();
    const int n_live = p.counters[0];
    const int n_tiles = n_live > 0 ? p.unit_start[n_live] : 0;
    if (static_cast<int>(blockIdx.x) >= n_tiles) return;     // uniform: before any barrier
    const PassEntry pe = p.passes[blockIdx.x];
    const int nbase = blockIdx.y * (KIND == 0 ? kGuCols : kBN);
    const int nk = p.kdim / kBK;
    const int n_chunks = (nk + kChunk - 1) / kChunk;

    if (tid == 0) {
        for (int i = 0; i < kAStages; ++i) {
            mbar_init(&S.full_a[i], 1);
            mbar_init(&S.mma_done[i], 1);
        }
        for (int i = 0; i < kBStages; ++i) mbar_init(&S.full_b[i], kDqWarps);   // one arrive per dequant warp
        for (int i = 0; i < 2; ++i) {
            mbar_init(&S.chunk_full[i], 1);
            mbar_init(&S.chunk_free[i], kFoldWarps);   // one arrive per fold warp
        }
        mbar_init(&S.done, 1);
        S.abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) tmem_alloc(&S.tmem_base, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem_base;
    volatile int* abort_flag = &S.abort_flag;
    int32_t* err = p.counters + 2;
    // stream bases: packed codes 16-byte aligned, scale / zero streams 8-byte aligned
    const bool ok_ptrs = pe.pk != 0 && pe.sc != 0 && (pe.pk & 15) == 0 && (pe.sc & 7) == 0 &&
                         (!ZERO || (pe.zp != 0 && (pe.zp & 7) == 0));
    if (!ok_ptrs && tid == 0) atomicOr(err, 1);

    if (warp < kDqWarps) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kDqRegs));
        // ── dequant producer: weight-tile row r = tid (KIND 0: rows 0-127 gate, 128-255 up of
        // intermediate rows nbase ..), all 64 codes of every stage (8 words; the two 32-code
        // halves may sit in different scale groups when the group is 32) ────────────────────
        const int r = tid;
        const int m = KIND == 0 ? (r >= kGuCols) : 0;
        const int row = KIND == 0 ? nbase + (r & (kGuCols - 1)) : nbase + r;
        const bool go = ok_ptrs && row < p.ndim;
        const uint32_t groups = static_cast<uint32_t>(p.kdim) >> p.gs_shift;
        const int32_t* src = reinterpret_cast<const int32_t*>(pe.pk) + p.w_off[m] + int64_t(row) * (p.kdim / 8);
        const uint32_t sidx0 = static_cast<uint32_t>(p.s_off[m]) + static_cast<uint32_t>(row) * groups;
        const uint32_t zidx0 = static_cast<uint32_t>(p.z_off[m]) + static_cast<uint32_t>(row >> 3) * groups;
        constexpr int kScLog = SC == VY_F32 ? 1 : 2;      // scale elements per 8-byte word: 2 or 4
        const int gs_shift = p.gs_shift;
        const int nib = 4 * (row & 7);
        WordStream<kScLog> scw;
        WordStream<1> zpw;
        scw.start(reinterpret_cast<const void*>(pe.sc), sidx0, sidx0 + groups - 1, go);
        if constexpr (ZERO) zpw.start(reinterpret_cast<const void*>(pe.zp), zidx0, zidx0 + groups - 1, go);
        // chunk c of tile row r sits at r * 128 + ((c ^ (r & 7)) << 4)
        const uint32_t sw = r & 7;
        unsigned char* b_base = reinterpret_cast<unsigned char*>(S.b[0]) + r * 128;
        auto issue = [&](int s) {
            if (s < nk && go) {
                cp_async16(&S.pack[s % kPack][0][tid], src + s * 8);
                cp_async16(&S.pack[s % kPack][1][tid], src + s * 8 + 4);
            }
            cp_async_commit();
        };
#pragma unroll
        for (int s = 0; s < kPack - 1; ++s) issue(s);
        for (int s = 0; s < nk; ++s) {
            issue(s + kPack - 1);
            uint32_t sp[2], bp[2];
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const uint32_t grp = static_cast<uint32_t>(s * kBK + hh * 32) >> gs_shift;
                const uint2 sw2 = scw.at(sidx0 + grp, go);
                sp[hh] = __byte_perm(scale_bits<ACT, SC>(sw2, (sidx0 + grp) & ((1u << kScLog) - 1)), 0, 0x1010);
                bp[hh] = int4_bias_pair<ACT>(8u);
                if constexpr (ZERO) {
                    const uint2 zw = zpw.at(zidx0 + grp, go);
                    bp[hh] = int4_bias_pair<ACT>(((((zidx0 + grp) & 1) ? zw.y : zw.x) >> nib) & 15u);
                }
            }
            cp_async_wait<kPack - 1>();
            const int slot = s % kBStages;
            // the slot is free once stage s - kBStages's MMAs are done; warp-uniform decision: a lane
            // that left the loop alone would strand the warp's arrive
            const int u = s - kBStages;
            if (u >= 0 &&
                !__all_sync(0xffffffffu, mbar_wait(&S.mma_done[u % kAStages], (u / kAStages) & 1, abort_flag, err)))
                break;
            const int ps = s % kPack;
            const uint4 w0 = S.pack[ps][0][tid], w1 = S.pack[ps][1][tid];
            const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
            unsigned char* dst = b_base + slot * (kBN * kBK * 2);
#pragma unroll
            for (int w = 0; w < 8; ++w) {
                const uint32_t bw = bp[w >> 2], spw = sp[w >> 2];
                uint4 o;
                o.x = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(words[w], 0), bw), spw);
                o.y = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(words[w], 1), bw), spw);
                o.z = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(words[w], 2), bw), spw);
                o.w = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(words[w], 3), bw), spw);
                *reinterpret_cast<uint4*>(dst + ((w ^ sw) << 4)) = o;
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.full_b[slot]);
        }
        cp_async_wait<0>();
    } else if (warp >= kCtlWarp) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kCtlRegs));
        if (warp == kCtlWarp && lane == 0) {
            // ── MMA issuer: nothing but the waits its MMAs need, the MMAs and one commit a stage
            // (the tensor core queues only a few MMAs: any other work here would let it drain) ─
            constexpr uint32_t idesc = idesc_f16<ACT>();
            for (int s = 0; s < nk; ++s) {
                const int sa = s % kAStages, sb = s % kBStages;
                const int c = s / kChunk, buf = c & 1, in_chunk = s - c * kChunk;
                // a chunk's buffer is free once the fold warps have read the chunk two before it
                if (in_chunk == 0 && c >= 2 &&
                    !mbar_wait(&S.chunk_free[buf], ((c >> 1) - 1) & 1, abort_flag, err))
                    break;
                if (!mbar_wait(&S.full_a[sa], (s / kAStages) & 1, abort_flag, err)) break;
                if (!mbar_wait(&S.full_b[sb], (s / kBStages) & 1, abort_flag, err)) break;
                tc_fence_after();
                const uint64_t ad = sw128_desc(S.a[sa]), bd = sw128_desc(S.b[sb]);
                const uint32_t d0 = tmem + buf * kBufCols;
#pragma unroll
                for (int j = 0; j < kBK / 16; ++j)   // K = 16 per instruction: +32 bytes per step
                    umma(d0, ad + 2 * j, bd + 2 * j, idesc, (in_chunk > 0 || j > 0) ? 1u : 0u);
                umma_commit(&S.mma_done[sa]);        // frees the activation and weight slots
                if (in_chunk == kChunk - 1 || s == nk - 1) umma_commit(&S.chunk_full[buf]);
            }
            umma_commit(&S.done);   // arrives once every MMA issued so far has completed
            // every MMA must be complete before TMEM is freed, on the abort path too
            mbar_drain(&S.done, 0, err);
        } else if (warp == kCtlWarp + 1 && lane == 0) {
            // ── activation producer: one TMA box per stage into the ring; a slot is refilled once
            // the MMAs of the stage that last used it are done ────────────────────────────────
            int loaded = 0;
            for (int t = 0; t < nk; ++t) {
                const int ts = t % kAStages, u = t - kAStages;
                if (u >= 0 && !mbar_wait(&S.mma_done[ts], (u / kAStages) & 1, abort_flag, err)) break;
                mbar_expect_tx(&S.full_a[ts], kTileBytes);
                tma_load_2d(S.a[ts], &tmap_a, t * kBK, pe.row0, &S.full_a[ts]);
                loaded = t + 1;
            }
            // every tile still in flight (only the last kAStages issued can be) lands before the
            // shared memory is released, on the abort path too
            for (int t = loaded > kAStages ? loaded - kAStages : 0; t < loaded; ++t)
                if (!mbar_drain(&S.full_a[t % kAStages], (t / kAStages) & 1, err)) break;
        }
        __syncwarp();
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kFoldRegs));
        // ── fold warps: warp f reads TMEM lanes 32 (f % 4) .. +31 (its lane quarter), column
        // quarter f / 4: KIND 0 gate columns [32 cq, +32) and the same up columns, KIND 1 down
        // columns [64 cq, +64) ──────────────────────────────────────────────────────────────
        const int f = warp - kDqWarps;
        const int q = f & 3, cq = f >> 2;
        const int m_row = q * 32 + lane;
        const uint32_t lane_addr = tmem + (uint32_t(q * 32) << 16);
        const int ncol0 = nbase + (KIND == 0 ? 32 * cq : 64 * cq);   // first output column
        const bool active = ncol0 < p.ndim;                        // warp-uniform
        auto col_of = [&](int i) {                                 // piece i: 8 columns
            return KIND == 0 ? ((i < 4) ? 32 * cq + 8 * i : kGuCols + 32 * cq + 8 * (i - 4)) : 64 * cq + 8 * i;
        };
        const bool live = m_row < pe.ncols;
        const int pos = pe.row0 + m_row;
        // KIND 1: the row's routing weight, fetched before the K loop (no epilogue latency)
        int rowid = 0;
        float wv = 0.f;
        if (KIND == 1 && active && live && ok_ptrs) {
            rowid = p.order[pos];
            const int64_t t = rowid / p.top_k;
            const int k = rowid - int(t) * p.top_k;
            const int widx = p.w_index ? p.w_index[rowid] : k;
            wv = load_as_float(p.weights, p.w_dtype, t * p.w_tok_stride + int64_t(widx) * p.w_slot_stride);
        }
        uint64_t acc[kFoldVals / 2];                               // fp32 pairs (columns 2j, 2j + 1)
        bool good = true;
        for (int c = 0; c < n_chunks; ++c) {
            const int buf = c & 1;
            if (!mbar_wait(&S.chunk_full[buf], (c >> 1) & 1, abort_flag, err)) {
                good = false;
                break;
            }
            tc_fence_after();
            if (active) {
                const uint32_t base = lane_addr + buf * kBufCols;
#pragma unroll
                for (int i = 0; i < kFoldVals / 8; ++i) {
                    uint32_t v[8];
                    tmem_ld8(base + col_of(i), v);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint64_t pv = pack_f32x2(v[2 * j], v[2 * j + 1]);
                        acc[4 * i + j] = c == 0 ? pv : add_f32x2(acc[4 * i + j], pv);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.chunk_free[buf]);
        }
        const bool finished = good && !*abort_flag && ok_ptrs;
        if (active && finished && live) {
            if constexpr (KIND == 0) {
                // h for intermediate columns ncol0 .. +32: four 8-element groups, each stored
                // permuted (and, on request, in natural order by row id) as soon as it is computed
                uint4* dst = reinterpret_cast<uint4*>(p.h_sorted + int64_t(pos) * p.ndim + ncol0);
                uint16_t* nat = p.h_out ? p.h_out + int64_t(p.order[pos]) * p.ndim + ncol0 : nullptr;
#pragma unroll
                for (int gq = 0; gq < 4; ++gq) {
                    uint32_t hg[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float2 gp = unpack_f32x2(acc[4 * gq + j / 2]), up = unpack_f32x2(acc[16 + 4 * gq + j / 2]);
                        const float gv = round_act<ACT>((j & 1) ? gp.y : gp.x);
                        const float uv = round_act<ACT>((j & 1) ? up.y : up.x);
                        const float av = round_act<ACT>(gv / (1.0f + expf(-gv)));
                        hg[j] = act_bits<ACT>(__fmul_rn(av, uv));
                    }
                    dst[gq] = make_uint4(hg[0] | (hg[4] << 16), hg[1] | (hg[5] << 16), hg[2] | (hg[6] << 16),
                                         hg[3] | (hg[7] << 16));
                    if (nat)
                        *reinterpret_cast<uint4*>(nat + 8 * gq) = make_uint4(
                            hg[0] | (hg[1] << 16), hg[2] | (hg[3] << 16), hg[4] | (hg[5] << 16), hg[6] | (hg[7] << 16));
                }
            } else {
                float4* dst = reinterpret_cast<float4*>(p.contrib + int64_t(rowid) * p.ndim + ncol0);
#pragma unroll
                for (int u = 0; u < kFoldVals / 4; ++u) {
                    float o[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float2 yp = unpack_f32x2(acc[2 * u + j / 2]);
                        float cv = __fmul_rn(round_act<ACT>((j & 1) ? yp.y : yp.x), wv);
                        if (p.w_round) cv = round_act<ACT>(cv);
                        o[j] = cv;
                    }
                    dst[u] = make_float4(o[0], o[1], o[2], o[3]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// The bounded barrier wait the GEMM kernels use, against a barrier that expects two arrivals and
// gets `arrivals`: with fewer, the wait runs out after `limit_ns`, sets error bit 4 and the kernel
// returns -- the failure path, exercised without a fault or a hang.
__global__ void selftest_wait_kernel(int arrivals, uint64_t limit_ns, int32_t* flags) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 2);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int i = 0; i < arrivals && i < 2; ++i) mbar_arrive(&bar);
        mbar_wait_for(&bar, 0, &abort_flag, flags, limit_ns);
    }
}

// ── host ────────────────────────────────────────────────────────────────────────────────────

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn(int* status) {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    *status = fn ? VY_OK : fail(VY_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    return fn;
}

// A [rows, cols] 16-bit matrix as 256 x 64 tiles with the 128-byte swizzle.
int make_tile_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int act) {
    int st;
    EncodeTiledFn fn = encode_fn(&st);
    if (!fn) return st;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
    const cuuint32_t box[2] = {kBK, kUnit};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, act == VY_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                    const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(VY_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return VY_OK;
}

struct PrefillLayout {
    int32_t *order, *live_expert, *live_start, *unit_start, *slot_order, *counters;
    PassEntry* passes;
    uint16_t *x_sorted, *h_sorted;
    float* contrib;
    size_t bytes;
    int64_t max_tiles;
};

PrefillLayout prefill_layout(const vy_moe_call* c, void* base) {
    const int64_t n = c->n_tokens * c->top_k, E = c->n_experts;
    const int64_t H = c->geom->hidden, I = c->geom->inter;
    Carve cv{static_cast<char*>(base), 0};
    PrefillLayout L{};
    L.order = cv.take<int32_t>(n);
    L.live_expert = cv.take<int32_t>(E);
    L.live_start = cv.take<int32_t>(E + 1);
    L.unit_start = cv.take<int32_t>(E + 1);
    L.slot_order = cv.take<int32_t>(n);
    L.counters = cv.take<int32_t>(4);
    L.max_tiles = n / kUnit + (n < E ? n : E) + 1;
    L.passes = cv.take<PassEntry>(L.max_tiles);
    L.x_sorted = cv.take<uint16_t>(n * H);
    L.h_sorted = cv.take<uint16_t>(n * I);
    L.contrib = c->contrib ? nullptr : cv.take<float>(n * H);
    L.bytes = cv.used;
    return L;
}

template <int ACT, int SC, bool ZERO, int KIND>
int launch_gemm(const CUtensorMap& map, const GemmParams& gp, int max_tiles, cudaStream_t s) {
    auto kern = gemm_kernel<ACT, SC, ZERO, KIND>;
    const size_t smem = sizeof(GemmSmem) + 1024;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return fail(VY_ERR_CUDA, "prefill GEMM shared memory: %s", cudaGetErrorString(e));
    // setmaxnreg.inc waits until the block's launch registers cover the split: never launch a
    // build whose register count would leave the fold warps waiting
    cudaFuncAttributes fa{};
    e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return fail(VY_ERR_CUDA, "prefill GEMM attributes: %s", cudaGetErrorString(e));
    if (static_cast<long long>(fa.numRegs) * kThreads < kRegSplit)
        return fail(VY_ERR_UNSUPPORTED, "prefill GEMM built with %d registers a thread: %d x %d < the %d its "
                    "register split needs", fa.numRegs, fa.numRegs, kThreads, kRegSplit);
    cudaLaunchConfig_t cfg = {};
    const int nblk = KIND == 0 ? gp.ndim / kGuCols : (gp.ndim + kBN - 1) / kBN;
    cfg.gridDim = dim3(static_cast<unsigned>(max_tiles), static_cast<unsigned>(nblk));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, map, gp);
    if (e != cudaSuccess) return fail(VY_ERR_CUDA, "prefill GEMM launch: %s", cudaGetErrorString(e));
    return VY_OK;
}

template <int ACT>
int dispatch_gemm(int kind, int sc, bool zero, const CUtensorMap& map, const GemmParams& gp, int max_tiles,
                  cudaStream_t s) {
#define VY_PF(SCV)                                                                                   \
    if (kind == 0)                                                                                   \
        return zero ? launch_gemm<ACT, SCV, true, 0>(map, gp, max_tiles, s)                          \
                    : launch_gemm<ACT, SCV, false, 0>(map, gp, max_tiles, s);                        \
    return zero ? launch_gemm<ACT, SCV, true, 1>(map, gp, max_tiles, s)                              \
                : launch_gemm<ACT, SCV, false, 1>(map, gp, max_tiles, s);
    switch (sc) {
        case VY_BF16: VY_PF(VY_BF16)
        case VY_F16: VY_PF(VY_F16)
        default: VY_PF(VY_F32)
    }
#undef VY_PF
}

int launch_prefill_gemm(int act, int kind, int sc, bool zero, const CUtensorMap& map, const GemmParams& gp,
                        int max_tiles, cudaStream_t s) {
    return act == VY_BF16 ? dispatch_gemm<VY_BF16>(kind, sc, zero, map, gp, max_tiles, s)
                          : dispatch_gemm<VY_F16>(kind, sc, zero, map, gp, max_tiles, s);
}

}  // namespace

int32_t* prefill_flags(const vy_moe_call* c) {
    char* base = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(c->workspace) + 1023) & ~uintptr_t(1023));
    return prefill_layout(c, base).counters + 2;
}

size_t prefill_workspace_bytes(const vy_moe_call* c) {
    if (!c || !c->geom) return 0;
    return prefill_layout(c, nullptr).bytes + 1024;
}

}  // namespace vy

using namespace vy;

extern "C" int vy_selftest_bounded_wait(int32_t arrivals, int64_t limit_ns, int32_t* flags, void* stream) {
    int st;
    if (!device_info(&st)) return st;
    if (!flags || limit_ns <= 0 || limit_ns > 2000000000ll)
        return fail(VY_ERR_INVALID, "flags %p, limit %lld ns (0, 2 s]", static_cast<void*>(flags), (long long)limit_ns);
    selftest_wait_kernel<<<1, 32, 0, as_stream(stream)>>>(arrivals, static_cast<uint64_t>(limit_ns), flags);
    return check_launch("vy_selftest_bounded_wait");
}

extern "C" int vy_moe_prefill(const vy_moe_call* c, void* stream) {
    int st;
    const DeviceInfo* dev = device_info(&st);
    if (!dev) return st;
    if ((st = validate_call(c)) != VY_OK) return st;
    if (c->n_tokens == 0) return ok();
    const vy_expert_geom& g = *c->geom;
    if (g.group_size < 32 || g.hidden % 128 || g.inter % kGuCols)
        return fail(VY_ERR_UNSUPPORTED, "prefill tiles need hidden / intermediate multiples of %d", kGuCols);
    // a stage's scale / zero element is read as the aligned 8-byte word holding it
    for (int r = 0; r < 3; ++r)
        if (g.scale_off[r] % (g.scale_dtype == VY_F32 ? 2 : 4) || (g.has_zero && g.zero_off[r] % 2))
            return fail(VY_ERR_UNSUPPORTED, "prefill: role %d's scale / zero offset is not a multiple of 8 bytes", r);
    if (c->h_out && !aligned16(c->h_out))
        return fail(VY_ERR_ALIGNMENT, "prefill: h_out must be 16-byte aligned");
    PrefillLayout L = prefill_layout(c, nullptr);
    if (!c->workspace || c->workspace_bytes < L.bytes + 1024)
        return fail(VY_ERR_WORKSPACE, "workspace %zu bytes, %zu needed", c->workspace_bytes, L.bytes + 1024);
    char* base = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(c->workspace) + 1023) & ~uintptr_t(1023));
    L = prefill_layout(c, base);
    cudaStream_t s = as_stream(stream);
    const int64_t n = c->n_tokens * c->top_k;
    int gs_shift = 0;
    while ((1 << gs_shift) < g.group_size) ++gs_shift;

    PlanArgs pa{};
    pa.ids = c->expert_ids;
    pa.ids64 = c->ids_dtype == VY_I64;
    pa.ids_stride = c->ids_row_stride ? c->ids_row_stride : c->top_k;
    pa.id_base = c->expert_base;
    pa.n_tokens = c->n_tokens;
    pa.top_k = c->top_k;
    pa.n_experts = c->n_experts;
    pa.order = L.order;
    pa.live_expert = L.live_expert;
    pa.live_start = L.live_start;
    pa.unit_start = L.unit_start;
    pa.slot_order = L.slot_order;
    pa.counters = L.counters;
    pa.tok_per_unit = kUnit;
    pa.expert_table = c->expert_table;
    pa.passes = L.passes;
    cudaEvent_t const* ev = reinterpret_cast<cudaEvent_t const*>(c->stage_events);
    const bool timed = ev != nullptr && c->n_stage_events >= 4;
    if (timed && cudaEventRecord(ev[0], s) != cudaSuccess)
        return fail(VY_ERR_INVALID, "stage_events[0] is not a usable cudaEvent_t");
    if ((st = launch_plan(pa, dev->sm_count, s)) != VY_OK) return st;

    GatherParams gp{c->x, c->x_row_stride, g.hidden, c->top_k, L.order, L.live_start, L.counters, L.x_sorted};
    {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>(dev->sm_count * 4));
        cfg.blockDim = dim3(256);
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaError_t e = cudaLaunchKernelEx(&cfg, gather_kernel, gp);
        if (e != cudaSuccess) return fail(VY_ERR_CUDA, "gather launch: %s", cudaGetErrorString(e));
    }

    CUtensorMap map_x, map_h;
    if ((st = make_tile_map(&map_x, L.x_sorted, n, g.hidden, c->act_dtype)) != VY_OK) return st;
    if ((st = make_tile_map(&map_h, L.h_sorted, n, g.inter, c->act_dtype)) != VY_OK) return st;

    GemmParams g1{};
    g1.kdim = g.hidden;
    g1.ndim = g.inter;
    g1.gs_shift = gs_shift;
    g1.top_k = c->top_k;
    g1.w_off[0] = g.word_off[0];
    g1.w_off[1] = g.word_off[1];
    g1.s_off[0] = g.scale_off[0];
    g1.s_off[1] = g.scale_off[1];
    g1.z_off[0] = g.zero_off[0];
    g1.z_off[1] = g.zero_off[1];
    g1.passes = L.passes;
    g1.unit_start = L.unit_start;
    g1.counters = L.counters;
    g1.order = L.order;
    g1.h_sorted = L.h_sorted;
    g1.h_out = static_cast<uint16_t*>(c->h_out);

    GemmParams g2 = g1;
    g2.kdim = g.inter;
    g2.ndim = g.hidden;
    g2.w_off[0] = g.word_off[2];
    g2.s_off[0] = g.scale_off[2];
    g2.z_off[0] = g.zero_off[2];
    g2.h_sorted = nullptr;
    g2.h_out = nullptr;
    g2.contrib = c->contrib ? c->contrib : L.contrib;
    g2.weights = c->weights;
    g2.w_dtype = c->w_dtype;
    g2.w_round = c->w_dtype == c->act_dtype;
    g2.w_tok_stride = c->w_tok_stride;
    g2.w_slot_stride = c->w_slot_stride;
    g2.w_index = c->w_index;

    const int max_tiles = static_cast<int>(L.max_tiles);
    const bool zero = g.has_zero != 0;
    if (timed) cudaEventRecord(ev[1], s);
    if ((st = launch_prefill_gemm(c->act_dtype, 0, g.scale_dtype, zero, map_x, g1, max_tiles, s)) != VY_OK)
        return st;
    if (timed) cudaEventRecord(ev[2], s);
    if ((st = launch_prefill_gemm(c->act_dtype, 1, g.scale_dtype, zero, map_h, g2, max_tiles, s)) != VY_OK)
        return st;
    if (timed && c->n_stage_events >= 5) cudaEventRecord(ev[4], s);
    if (c->contrib) {
        if (timed) cudaEventRecord(ev[3], s);
        return check_launch("vy_moe_prefill");
    }
    if ((st = launch_layer_combine(c, L.contrib, L.slot_order, s)) != VY_OK) return st;
    if (timed) cudaEventRecord(ev[3], s);
    return check_launch("vy_moe_prefill");
}
