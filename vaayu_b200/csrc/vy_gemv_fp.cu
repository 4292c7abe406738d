// vy_gemv_fp.cu -- FP8-e4m3 / FP4-e2m1 block-scaled dequant fused into a decode GEMV
// (batch <= 16): y[t, n] = bf16(sum_k deq(W)[n, k] * x[t, k]), fp32 accumulation.
//
// One CTA = 16 weight rows; its 16 warps split K into 16 contiguous ranges (split-K inside the
// CTA, so the grid has n/16 CTAs even for a single output tile row; two CTAs fit an SM at 64
// registers a thread).  Each warp streams its range through its own cp.async ring in shared
// memory, dequantises into bf16 pairs in registers (exactly the values vy_fp8_dequant /
// vy_fp4_dequant produce) and accumulates m16n8k16 tensor-core fragments whose N dimension is
// the tokens.  The partial tiles are summed in warp order in
// shared memory: the result does not depend on scheduling.
#include <cuda_fp8.h>

#include "vy_common.cuh"

namespace vy {
namespace {

#ifndef VY_GEMV_WARPS
#define VY_GEMV_WARPS 16
#endif
#ifndef VY_GEMV_DEPTH
#define VY_GEMV_DEPTH 4
#endif
constexpr int kWarps = VY_GEMV_WARPS;   // warps per CTA: the K split of one 16-row tile
constexpr int kDepth = VY_GEMV_DEPTH;   // ring steps per warp (1 KB each; kDepth - 1 in flight)

__device__ __forceinline__ float e4m3f(uint32_t b) {
    __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(b & 0xFFu), __NV_E4M3);
    return __half2float(__half(h));
}

// Two e4m3 codes (the low 16 bits of `b`) as floats, exactly.
__device__ __forceinline__ float2 e4m3x2f(uint32_t b) {
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(b & 0xFFFFu), __NV_E4M3);
    return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

// Four e2m1 codes (bits 0-15, low nibble first) as two bf16 pairs, exactly: each byte to an f16
// pair by the hardware conversion, widened to fp32 and narrowed to bf16 (e2m1 values are 0, 0.5
// .. 6, exact in all three).
__device__ __forceinline__ void e2m1x4_bf16(uint32_t c, uint32_t& e01, uint32_t& e23) {
    const uint32_t h0 = e2m1x2_f16(c), h1 = e2m1x2_f16(c >> 8);
    const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&h0));
    const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&h1));
    const __nv_bfloat162 p0 = __floats2bfloat162_rn(f0.x, f0.y), p1 = __floats2bfloat162_rn(f1.x, f1.y);
    e01 = *reinterpret_cast<const uint32_t*>(&p0);
    e23 = *reinterpret_cast<const uint32_t*>(&p1);
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ float e2m1f(uint32_t nib) {
    uint32_t e = (nib >> 1) & 3u, m = nib & 1u;
    uint32_t bits = e ? (((e + 126u) << 23) | (m << 22)) : (m ? 0x3F000000u : 0u);
    return __uint_as_float(bits | ((nib & 8u) << 28));
}

__device__ __forceinline__ float block_scale(const void* p, int dtype, int64_t i) {
    switch (dtype) {
        case VY_F32: return __ldg(reinterpret_cast<const float*>(p) + i);
        case VY_BF16: return __bfloat162float(__ldg(reinterpret_cast<const __nv_bfloat16*>(p) + i));
        case VY_F16: return __half2float(__ldg(reinterpret_cast<const __half*>(p) + i));
        default: {
            uint8_t b = __ldg(reinterpret_cast<const uint8_t*>(p) + i);
            if (b == 0xFF) return __int_as_float(0x7FC00000);
            if (b == 0) return 5.877471754111438e-39f;
            return __int_as_float(static_cast<int>(b) << 23);
        }
    }
}

__device__ __forceinline__ uint32_t bf16_pair(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

struct GemvParams {
    const uint8_t* w;
    int64_t n, k;
    const void* scale;
    int scale_dtype;
    int64_t srows, scols, bo, bi;   // fp8 block scales
    int gs;                         // fp4 group
    int div_shift;                  // log2 of the fp8 block width / fp4 group when a power of two, else -1
    const __nv_bfloat16* x;
    int64_t x_stride;
    int n_tokens;
    __nv_bfloat16* out;
    int64_t out_stride;
};

// KIND 0: fp8 (16 B = 16 codes of a row per thread per step; a step covers 64 K per row)
// KIND 1: fp4 (16 B = 32 codes; a step covers 128 K per row)
// Each warp streams its K range through its own cp.async ring in shared memory (kDepth steps of
// 1 KB: rows g and g + 8 of the tile, 16 B per lane each), kDepth - 1 steps ahead of the math.
// SC: the fp8 block scales' dtype, fixed at compile time (no per-step dispatch).
template <int KIND, int NB, int SC>
__global__ void __launch_bounds__(kWarps * 32, kWarps >= 16 ? 2 : 1) fp_gemv_kernel(GemvParams p) {
    constexpr int kPerThread = KIND == 0 ? 16 : 32;    // K elements per thread per step
    constexpr int kStepK = 4 * kPerThread;             // K per step per row
    extern __shared__ uint4 gv_ring[];                 // [kWarps][kDepth][2][32]
    __shared__ float part[kWarps][16][NB * 8];
    grid_dependency_wait();      // launched chained to the previous kernel on the stream
    grid_dependents_launch();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, tig = lane & 3;
    uint4* my_ring = gv_ring + warp * (kDepth * 64);
    const int64_t row0 = int64_t(blockIdx.x) * 16;
    const int64_t steps = p.k / kStepK;
    const int64_t per_warp = (steps + kWarps - 1) / kWarps;
    const int64_t s_lo = warp * per_warp, s_hi = min(steps, s_lo + per_warp);
    const int64_t rA = row0 + g, rB = row0 + g + 8;
    const bool okA = rA < p.n, okB = rB < p.n;
    const int64_t row_bytes = KIND == 0 ? p.k : p.k / 2;
    const uint8_t* wA = p.w + (okA ? rA : 0) * row_bytes;
    const uint8_t* wB = p.w + (okB ? rB : 0) * row_bytes;
    // per-row scale bases, and K -> block / group index with a shift when possible (32-bit: k < 2^31)
    const int64_t baseA = KIND == 0 ? (okA ? (rA / p.bo) * p.scols : 0) : (okA ? rA * (p.k / p.gs) : 0);
    const int64_t baseB = KIND == 0 ? (okB ? (rB / p.bo) * p.scols : 0) : (okB ? rB * (p.k / p.gs) : 0);
    const uint32_t div = static_cast<uint32_t>(KIND == 0 ? p.bi : p.gs);
    const int dsh = p.div_shift;
    auto kdiv = [&](uint32_t kk) { return dsh >= 0 ? (kk >> dsh) : (kk / div); };
    const bool halves = KIND == 1 && (p.gs % 16) == 0;   // a thread's 32 fp4 codes: two whole groups
    const uint8_t* sc8 = reinterpret_cast<const uint8_t*>(p.scale);

    // ── issue side: one step (rows A and B, 16 B per lane each) per call ──────────────────
    int64_t i_s = s_lo;
    int i_slot = 0;
    constexpr int kStepBytes = KIND == 0 ? kStepK : kStepK / 2;
    const uint8_t* srcA = wA + (s_lo * kStepK + tig * kPerThread) / (KIND == 0 ? 1 : 2);
    const uint8_t* srcB = wB + (s_lo * kStepK + tig * kPerThread) / (KIND == 0 ? 1 : 2);
    auto issue = [&]() {
        if (i_s < s_hi) {
            uint4* dst = my_ring + i_slot * 64 + lane;
            if (okA) cp_async16(dst, srcA);
            if (okB) cp_async16(dst + 32, srcB);
            srcA += kStepBytes;
            srcB += kStepBytes;
        }
        cp_async_commit();
        ++i_s;
        if (++i_slot == kDepth) i_slot = 0;
    };
#pragma unroll
    for (int d = 0; d < kDepth - 1; ++d) issue();

    // this lane's token column in each block (null past the batch), at its K offset in a step
    const __nv_bfloat16* xrow[NB];
#pragma unroll
    for (int cb = 0; cb < NB; ++cb)
        xrow[cb] = cb * 8 + g < p.n_tokens ? p.x + int64_t(cb * 8 + g) * p.x_stride + tig * kPerThread : nullptr;

    float acc[NB][4];
#pragma unroll
    for (int cb = 0; cb < NB; ++cb)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[cb][i] = 0.f;

    int c_slot = 0;
    for (int64_t s = s_lo; s < s_hi; ++s) {
        issue();
        cp_async_wait<kDepth - 1>();
        const uint4* st = my_ring + c_slot * 64 + lane;
        const uint4 va = okA ? st[0] : make_uint4(0u, 0u, 0u, 0u);
        const uint4 vb = okB ? st[32] : make_uint4(0u, 0u, 0u, 0u);
        if (++c_slot == kDepth) c_slot = 0;
        const uint32_t k0 = static_cast<uint32_t>(s * kStepK + tig * kPerThread);
        float sa = 0.f, sb = 0.f;
        uint32_t ha[2] = {0u, 0u}, hb[2] = {0u, 0u};   // fp4 group scales as bf16 pairs (exact)
        if constexpr (KIND == 0) {
            const uint32_t kb = kdiv(k0);
            sa = okA ? block_scale(p.scale, SC, baseA + kb) : 0.f;
            sb = okB ? block_scale(p.scale, SC, baseB + kb) : 0.f;
        } else if (halves) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const uint32_t gi = kdiv(k0 + 16 * hh);
                ha[hh] = okA ? bf16_pair(e4m3f(__ldg(sc8 + baseA + gi)), e4m3f(__ldg(sc8 + baseA + gi))) : 0u;
                hb[hh] = okB ? bf16_pair(e4m3f(__ldg(sc8 + baseB + gi)), e4m3f(__ldg(sc8 + baseB + gi))) : 0u;
            }
        }
        const uint32_t wa[4] = {va.x, va.y, va.z, va.w};
        const uint32_t wb[4] = {vb.x, vb.y, vb.z, vb.w};
        // mma step q covers this thread's elements 4q..4q+3 (fp8) / 4q..4q+3 (fp4)
        constexpr int kSteps = kPerThread / 4;
#pragma unroll
        for (int q = 0; q < kSteps; ++q) {
            uint32_t a0, a1, a2, a3;
            if constexpr (KIND == 0) {
                const uint32_t xa = wa[q], xb = wb[q];   // 4 codes: elements 4q..4q+3
                const float2 fa0 = e4m3x2f(xa), fa1 = e4m3x2f(xa >> 16);
                const float2 fb0 = e4m3x2f(xb), fb1 = e4m3x2f(xb >> 16);
                a0 = bf16_pair(__fmul_rn(fa0.x, sa), __fmul_rn(fa0.y, sa));
                a2 = bf16_pair(__fmul_rn(fa1.x, sa), __fmul_rn(fa1.y, sa));
                a1 = bf16_pair(__fmul_rn(fb0.x, sb), __fmul_rn(fb0.y, sb));
                a3 = bf16_pair(__fmul_rn(fb1.x, sb), __fmul_rn(fb1.y, sb));
            } else {
                const uint32_t xa = (wa[q >> 1] >> (16 * (q & 1))) & 0xFFFFu;   // 4 nibbles
                const uint32_t xb = (wb[q >> 1] >> (16 * (q & 1))) & 0xFFFFu;
                if (halves) {
                    // e2m1 x e4m3 has at most 6 significant bits: the bf16 product is exact,
                    // i.e. the same value the fp32 product rounded to bf16 gives
                    uint32_t ea01, ea23, eb01, eb23;
                    e2m1x4_bf16(xa, ea01, ea23);
                    e2m1x4_bf16(xb, eb01, eb23);
                    a0 = bf16x2_mul(ea01, ha[q >> 2]);
                    a2 = bf16x2_mul(ea23, ha[q >> 2]);
                    a1 = bf16x2_mul(eb01, hb[q >> 2]);
                    a3 = bf16x2_mul(eb23, hb[q >> 2]);
                } else {
                    const uint32_t gi = kdiv(k0 + 4 * q);
                    const float fa = okA ? e4m3f(__ldg(sc8 + baseA + gi)) : 0.f;
                    const float fb = okB ? e4m3f(__ldg(sc8 + baseB + gi)) : 0.f;
                    a0 = bf16_pair(__fmul_rn(e2m1f(xa), fa), __fmul_rn(e2m1f(xa >> 4), fa));
                    a2 = bf16_pair(__fmul_rn(e2m1f(xa >> 8), fa), __fmul_rn(e2m1f(xa >> 12), fa));
                    a1 = bf16_pair(__fmul_rn(e2m1f(xb), fb), __fmul_rn(e2m1f(xb >> 4), fb));
                    a3 = bf16_pair(__fmul_rn(e2m1f(xb >> 8), fb), __fmul_rn(e2m1f(xb >> 12), fb));
                }
            }
#pragma unroll
            for (int cb = 0; cb < NB; ++cb) {
                uint2 xv = make_uint2(0u, 0u);
                if (xrow[cb]) xv = *reinterpret_cast<const uint2*>(xrow[cb] + s * kStepK + 4 * q);
                mma_16816<VY_BF16>(acc[cb], a0, a1, a2, a3, xv.x, xv.y);
            }
        }
    }
    cp_async_wait<0>();
#pragma unroll
    for (int cb = 0; cb < NB; ++cb)
#pragma unroll
        for (int i = 0; i < 4; ++i) part[warp][g + 8 * (i >> 1)][cb * 8 + 2 * tig + (i & 1)] = acc[cb][i];
    __syncthreads();
    for (int idx = threadIdx.x; idx < 16 * NB * 8; idx += blockDim.x) {
        const int r = idx / (NB * 8), t = idx % (NB * 8);
        float a = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) a += part[w][r][t];
        if (t < p.n_tokens && row0 + r < p.n)
            p.out[int64_t(t) * p.out_stride + row0 + r] = __float2bfloat16_rn(a);
    }
}

constexpr size_t kRingBytes = size_t(kWarps) * kDepth * 64 * sizeof(uint4);

// ── single-token NVFP4: f16 tensor-core operands ─────────────────────────────────────────
//
// One token (decode at batch 1) takes fp4_t1_kernel: the grid and the K split of fp_gemv_kernel,
// with the arithmetic in f16.  cvt.rn.f16x2.e2m1x2 turns a byte (two codes) into an f16 pair, and
// the product with the e4m3 group scale is exact in f16 (at most 6 significant bits, magnitudes
// 2^-10 .. 2688), so the weights equal the bf16 dequantised ones.  Each warp stages its K range
// of the activations in shared memory as x * 2^-s, s chosen so the range's largest |x| lands in
// [2^14, 2^15): a bf16 value (8 significant bits) converts to f16 exactly down to 2^-28 of that
// largest magnitude.  The warp's partial dots are multiplied back by 2^s (exact), so products
// and sums equal those of the bf16 operands.  (A range whose largest |x| is below 2^-112 is staged
// with s = -126 and loses low bits; an infinite or NaN activation is staged unscaled.)  A code
// costs half a conversion and half an f16 multiply, against the multi-token kernel's conversion,
// widening and narrowing to bf16 and bf16 multiply.

#ifndef VY_GEMV_T1_WARPS
#define VY_GEMV_T1_WARPS 16
#endif
constexpr int kT1Warps = VY_GEMV_T1_WARPS;
constexpr int kT1StepK = 128;                     // K per step per row (16 B of codes a lane)
constexpr size_t kT1RingBytes = size_t(kT1Warps) * kDepth * 64 * sizeof(uint4);

// Four bytes of e2m1 codes (eight values, low nibble first) as four f16 pairs.
__device__ __forceinline__ void e2m1x8_f16(uint32_t c, uint32_t& d0, uint32_t& d1, uint32_t& d2, uint32_t& d3) {
    d0 = e2m1x2_f16(c);
    d1 = e2m1x2_f16(c >> 8);
    d2 = e2m1x2_f16(c >> 16);
    d3 = e2m1x2_f16(c >> 24);
}

// Two e4m3 codes (bits 0-15, first in the low byte) as an f16 pair (exact).
__device__ __forceinline__ uint32_t e4m3x2_f16(uint32_t b) {
    uint32_t d;
    asm("{ .reg .b16 h; cvt.u16.u32 h, %1; cvt.rn.f16x2.e4m3x2 %0, h; }" : "=r"(d) : "r"(b));
    return d;
}

__device__ __forceinline__ uint32_t f16x2_mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// The staging exponent s of a range whose largest |x| is m (see above).
__device__ __forceinline__ int stage_shift(float m) {
    if (!(m > 0.f) || !(m < __int_as_float(0x7F800000))) return 0;   // zero, infinite or NaN: unscaled
    const int field = __float_as_int(m) >> 23;                        // biased exponent (m > 0)
    const int s = field == 0 ? -126 : field - 127 - 14;
    return s < -126 ? -126 : s;
}
__device__ __forceinline__ float pow2f(int s) {   // 2^s for s in [-126, 127]
    return __int_as_float((s + 127) << 23);
}

// G16: 16-code groups with 2-byte aligned scale rows -- one 16-bit load brings a row's two group
// scales of a step.
template <bool G16>
__global__ void __launch_bounds__(kT1Warps * 32, 32 / kT1Warps) fp4_t1_kernel(GemvParams p) {
    extern __shared__ uint4 t1_ring[];             // [kT1Warps][kDepth][2][32], then the staged x
    __shared__ float part[kT1Warps][16];
    grid_dependency_wait();
    grid_dependents_launch();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, tig = lane & 3;
    uint4* my_ring = t1_ring + warp * (kDepth * 64);
    const int64_t row0 = int64_t(blockIdx.x) * 16;
    const int64_t steps = p.k / kT1StepK;
    const int64_t s_lo = warp * steps / kT1Warps, s_hi = (warp + 1) * steps / kT1Warps;
    const int64_t rA = row0 + g, rB = row0 + g + 8;
    const bool okA = rA < p.n, okB = rB < p.n;
    const uint8_t* wA = p.w + (okA ? rA : 0) * (p.k / 2);
    const uint8_t* wB = p.w + (okB ? rB : 0) * (p.k / 2);
    const uint8_t* sA = reinterpret_cast<const uint8_t*>(p.scale) + (okA ? rA : 0) * (p.k / p.gs);
    const uint8_t* sB = reinterpret_cast<const uint8_t*>(p.scale) + (okB ? rB : 0) * (p.k / p.gs);
    const uint32_t div = static_cast<uint32_t>(p.gs);
    const int dsh = p.div_shift;
    auto kdiv = [&](uint32_t kk) { return dsh >= 0 ? (kk >> dsh) : (kk / div); };

    int64_t i_s = s_lo;
    int i_slot = 0;
    const uint8_t* srcA = wA + (s_lo * kT1StepK + tig * 32) / 2;   // this lane's 16 bytes of the next step
    const uint8_t* srcB = wB + (s_lo * kT1StepK + tig * 32) / 2;
    auto issue = [&]() {
        if (i_s < s_hi) {
            uint4* dst = my_ring + i_slot * 64 + lane;
            if (okA) cp_async16(dst, srcA);
            if (okB) cp_async16(dst + 32, srcB);
            srcA += kT1StepK / 2;
            srcB += kT1StepK / 2;
        }
        cp_async_commit();
        ++i_s;
        if (++i_slot == kDepth) i_slot = 0;
    };
#pragma unroll
    for (int d = 0; d < kDepth - 1; ++d) issue();

    // stage this warp's activations: x * 2^-sh as f16
    const int64_t max_len = ((steps + kT1Warps - 1) / kT1Warps) * kT1StepK;
    __half* xs = reinterpret_cast<__half*>(t1_ring + kT1Warps * kDepth * 64) + warp * max_len;
    const int64_t len = (s_hi - s_lo) * kT1StepK;
    const __nv_bfloat16* xt = p.x + s_lo * kT1StepK;
    float m = 0.f;
    for (int64_t k = 4 * lane; k < len; k += 128) {
        const uint2 v = *reinterpret_cast<const uint2*>(xt + k);
        m = fmaxf(m, fmaxf(fmaxf(fabsf(__uint_as_float(v.x << 16)), fabsf(__uint_as_float(v.x & 0xFFFF0000u))),
                           fmaxf(fabsf(__uint_as_float(v.y << 16)), fabsf(__uint_as_float(v.y & 0xFFFF0000u)))));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    const int sh = stage_shift(m);
    const float down = pow2f(-sh);
    for (int64_t k = 4 * lane; k < len; k += 128) {
        const uint2 v = *reinterpret_cast<const uint2*>(xt + k);
        const __half2 h0 = __floats2half2_rn(__uint_as_float(v.x << 16) * down, __uint_as_float(v.x & 0xFFFF0000u) * down);
        const __half2 h1 = __floats2half2_rn(__uint_as_float(v.y << 16) * down, __uint_as_float(v.y & 0xFFFF0000u) * down);
        *reinterpret_cast<uint2*>(xs + k) = make_uint2(*reinterpret_cast<const uint32_t*>(&h0),
                                                       *reinterpret_cast<const uint32_t*>(&h1));
    }
    __syncwarp();

    // the group scales of step i (rows A and B, groups of codes 0-15 and 16-31), loaded a step early
    auto load_scales = [&](int64_t i, uint32_t& ga, uint32_t& gb) {
        ga = gb = 0u;
        if (i >= s_hi) return;
        if constexpr (G16) {
            const int64_t g0 = i * (kT1StepK / 16) + tig * 2;
            if (okA) ga = __ldg(reinterpret_cast<const unsigned short*>(sA + g0));
            if (okB) gb = __ldg(reinterpret_cast<const unsigned short*>(sB + g0));
        } else {
            const uint32_t k0 = static_cast<uint32_t>(i * kT1StepK + tig * 32);
            const uint32_t g0 = kdiv(k0), g1 = kdiv(k0 + 16);
            if (okA) ga = __ldg(sA + g0) | (uint32_t(__ldg(sA + g1)) << 8);
            if (okB) gb = __ldg(sB + g0) | (uint32_t(__ldg(sB + g1)) << 8);
        }
    };
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int c_slot = 0;
    uint32_t ga, gb;
    load_scales(s_lo, ga, gb);
    for (int64_t s = s_lo; s < s_hi; ++s) {
        uint32_t na, nb;
        load_scales(s + 1, na, nb);
        issue();
        cp_async_wait<kDepth - 1>();
        const uint4* st = my_ring + c_slot * 64 + lane;
        const uint4 va = okA ? st[0] : make_uint4(0u, 0u, 0u, 0u);
        const uint4 vb = okB ? st[32] : make_uint4(0u, 0u, 0u, 0u);
        if (++c_slot == kDepth) c_slot = 0;
        const uint32_t wa[4] = {va.x, va.y, va.z, va.w};
        const uint32_t wb[4] = {vb.x, vb.y, vb.z, vb.w};
        // the two groups' scales as f16 pairs holding each twice (exact)
        const uint32_t pa = e4m3x2_f16(ga), pb = e4m3x2_f16(gb);
        const uint32_t ha[2] = {__byte_perm(pa, 0, 0x1010), __byte_perm(pa, 0, 0x3232)};
        const uint32_t hb[2] = {__byte_perm(pb, 0, 0x1010), __byte_perm(pb, 0, 0x3232)};
        const __half* xq = xs + (s - s_lo) * kT1StepK + tig * 32;
#pragma unroll
        for (int j = 0; j < 4; ++j) {      // word j: codes 8j .. 8j + 7 = mma steps 2j, 2j + 1
            uint32_t ea[4], eb[4];
            e2m1x8_f16(wa[j], ea[0], ea[1], ea[2], ea[3]);
            e2m1x8_f16(wb[j], eb[0], eb[1], eb[2], eb[3]);
            const uint32_t sa = ha[j >> 1], sb = hb[j >> 1];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint2 xv = make_uint2(0u, 0u);
                if (g == 0) xv = *reinterpret_cast<const uint2*>(xq + 8 * j + 4 * h);
                mma_16816<VY_F16>(acc, f16x2_mul(ea[2 * h], sa), f16x2_mul(eb[2 * h], sb),
                                  f16x2_mul(ea[2 * h + 1], sa), f16x2_mul(eb[2 * h + 1], sb), xv.x, xv.y);
            }
        }
        ga = na;
        gb = nb;
    }
    cp_async_wait<0>();
    // column 0 of the fragment is the token: acc[0] row g, acc[2] row g + 8 (lanes with tig 0)
    if (tig == 0) {
        const float up = pow2f(sh);
        part[warp][g] = acc[0] * up;
        part[warp][g + 8] = acc[2] * up;
    }
    __syncthreads();
    if (threadIdx.x < 16) {
        float a = 0.f;
#pragma unroll
        for (int w = 0; w < kT1Warps; ++w) a += part[w][threadIdx.x];
        if (row0 + threadIdx.x < p.n) p.out[row0 + threadIdx.x] = __float2bfloat16_rn(a);
    }
}

size_t t1_smem(int64_t k) {
    const int64_t steps = k / kT1StepK;
    return kT1RingBytes + size_t((steps + kT1Warps - 1) / kT1Warps) * kT1StepK * kT1Warps * 2;
}

// The largest dynamic shared memory fp4_t1_kernel may take on this device (its limit is raised to
// that once per device; 0 when the setup failed).
template <bool G16>
size_t t1_smem_limit() {
    static size_t limit[kMaxDevices] = {};
    const int st = once_per_device(
        reinterpret_cast<const void*>(fp4_t1_kernel<G16>),
        [](int dev, void*) -> int {
            cudaFuncAttributes fa;
            int optin = 0;
            if (cudaFuncGetAttributes(&fa, fp4_t1_kernel<G16>) != cudaSuccess ||
                cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
                return VY_ERR_CUDA;
            const int room = optin - static_cast<int>(fa.sharedSizeBytes);
            if (room <= 0 || cudaFuncSetAttribute(fp4_t1_kernel<G16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  room) != cudaSuccess)
                return VY_ERR_CUDA;
            limit[dev] = static_cast<size_t>(room);
            return VY_OK;
        },
        nullptr);
    const int d = current_device();
    return (st == VY_OK && d >= 0 && d < kMaxDevices) ? limit[d] : 0;
}

template <int KIND, int NB, int SC>
cudaError_t launch_one(unsigned grid, const GemvParams& p, cudaStream_t s) {
    const int st = once_per_device(
        reinterpret_cast<const void*>(fp_gemv_kernel<KIND, NB, SC>),
        [](int, void*) -> int {
            return cudaFuncSetAttribute(fp_gemv_kernel<KIND, NB, SC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(kRingBytes)) == cudaSuccess ? VY_OK : VY_ERR_CUDA;
        },
        nullptr);
    if (st != VY_OK) return cudaErrorInvalidValue;
    return launch_chained(fp_gemv_kernel<KIND, NB, SC>, dim3(grid), dim3(kWarps * 32), kRingBytes, s, p);
}

// FP8 launches by block-scale dtype (SC is the first candidate tried).
template <int SC>
cudaError_t launch_fp8(int sc, bool two, unsigned grid, const GemvParams& p, cudaStream_t s) {
    if (sc == SC || SC == VY_E8M0)
        return two ? launch_one<0, 2, SC>(grid, p, s) : launch_one<0, 1, SC>(grid, p, s);
    if constexpr (SC == VY_F32) return launch_fp8<VY_BF16>(sc, two, grid, p, s);
    else if constexpr (SC == VY_BF16) return launch_fp8<VY_F16>(sc, two, grid, p, s);
    else return launch_fp8<VY_E8M0>(sc, two, grid, p, s);
}

// One-token NVFP4 calls with whole 16-code groups take fp4_t1_kernel while its staged activations
// fit in shared memory; the rest fp_gemv_kernel.
int launch_gemv(int kind, const GemvParams& p, cudaStream_t s) {
    const unsigned grid = static_cast<unsigned>((p.n + 15) / 16);
    const bool two = p.n_tokens > 8;
    cudaError_t e;
    const size_t t1 = kind == 1 && p.n_tokens == 1 && p.gs % 16 == 0 ? t1_smem(p.k) : 0;
    const bool g16 = p.gs == 16 && (reinterpret_cast<uintptr_t>(p.scale) & 1u) == 0 && (p.k / 16) % 2 == 0;
    if (t1 && g16 && t1 <= t1_smem_limit<true>())
        e = launch_chained(fp4_t1_kernel<true>, dim3(grid), dim3(kT1Warps * 32), t1, s, p);
    else if (t1 && !g16 && t1 <= t1_smem_limit<false>())
        e = launch_chained(fp4_t1_kernel<false>, dim3(grid), dim3(kT1Warps * 32), t1, s, p);
    else
        e = kind == 1 ? (two ? launch_one<1, 2, VY_E4M3>(grid, p, s) : launch_one<1, 1, VY_E4M3>(grid, p, s))
                      : launch_fp8<VY_F32>(p.scale_dtype, two, grid, p, s);
    if (e != cudaSuccess) return fail(VY_ERR_CUDA, "%s launch: %s", kind == 0 ? "vy_fp8_gemv" : "vy_fp4_gemv",
                                      cudaGetErrorString(e));
    return check_launch(kind == 0 ? "vy_fp8_gemv" : "vy_fp4_gemv");
}

int pow2_shift(int64_t v) {
    if (v <= 0 || (v & (v - 1))) return -1;
    int s = 0;
    while ((int64_t(1) << s) < v) ++s;
    return s;
}

int common_checks(const uint8_t* w, int64_t n, int64_t k, const void* x, int64_t x_stride,
                  int64_t n_tokens, void* out, int64_t out_stride, int64_t step) {
    if (n < 0 || k < 0 || n_tokens < 0) return fail(VY_ERR_INVALID, "negative size");
    if (k >= (int64_t(1) << 31)) return fail(VY_ERR_UNSUPPORTED, "k %lld >= 2^31", (long long)k);
    if (n_tokens > 16) return fail(VY_ERR_UNSUPPORTED, "batch %lld > 16", (long long)n_tokens);
    if (k % step) return fail(VY_ERR_UNSUPPORTED, "k %lld is not a multiple of %lld", (long long)k, (long long)step);
    if (n == 0 || n_tokens == 0) return VY_OK;
    if (!w || !x || !out) return fail(VY_ERR_INVALID, "null pointer");
    if (!aligned16(w)) return fail(VY_ERR_ALIGNMENT, "weight not 16-byte aligned");
    if ((reinterpret_cast<uintptr_t>(x) & 7u) || (x_stride % 4))
        return fail(VY_ERR_ALIGNMENT, "x must be 8-byte aligned with a row stride multiple of 4");
    if (x_stride < k || out_stride < n) return fail(VY_ERR_INVALID, "row stride too small");
    return VY_OK;
}

}  // namespace
}  // namespace vy

using namespace vy;

extern "C" int vy_fp8_gemv(const uint8_t* w, int64_t n, int64_t k, const void* scale,
                           int32_t scale_dtype, int64_t srows, int64_t scols, const void* x,
                           int64_t x_stride, int64_t n_tokens, void* out, int64_t out_stride,
                           void* stream) {
    int st;
    const DeviceInfo* dev = device_info(&st);
    if (!dev) return st;
    if ((st = common_checks(w, n, k, x, x_stride, n_tokens, out, out_stride, 64)) != VY_OK) return st;
    if (n == 0 || n_tokens == 0) return ok();
    if (srows <= 0 || scols <= 0 || n % srows || k % scols)
        return fail(VY_ERR_INVALID, "scale [%lld, %lld] does not tile [%lld, %lld]", (long long)srows,
                    (long long)scols, (long long)n, (long long)k);
    if ((k / scols) % 16) return fail(VY_ERR_UNSUPPORTED, "fp8 block width %lld (multiple of 16)", (long long)(k / scols));
    if (scale_dtype != VY_F32 && scale_dtype != VY_BF16 && scale_dtype != VY_F16 && scale_dtype != VY_E8M0)
        return fail(VY_ERR_UNSUPPORTED, "block-scale dtype %d", scale_dtype);
    if (!scale) return fail(VY_ERR_INVALID, "null scale");
    GemvParams p{w, n, k, scale, scale_dtype, srows, scols, n / srows, k / scols, 0, pow2_shift(k / scols),
                 reinterpret_cast<const __nv_bfloat16*>(x), x_stride, static_cast<int>(n_tokens),
                 reinterpret_cast<__nv_bfloat16*>(out), out_stride};
    return launch_gemv(0, p, as_stream(stream));
}

extern "C" int vy_fp4_gemv(const uint8_t* w, int64_t n, int64_t k, const uint8_t* scale,
                           int32_t group_size, const void* x, int64_t x_stride, int64_t n_tokens,
                           void* out, int64_t out_stride, void* stream) {
    int st;
    const DeviceInfo* dev = device_info(&st);
    if (!dev) return st;
    if ((st = common_checks(w, n, k, x, x_stride, n_tokens, out, out_stride, 128)) != VY_OK) return st;
    if (n == 0 || n_tokens == 0) return ok();
    if (group_size <= 0 || group_size % 4 || k % group_size)
        return fail(VY_ERR_UNSUPPORTED, "fp4 group %d", group_size);
    if (!scale) return fail(VY_ERR_INVALID, "null scale");
    GemvParams p{w, n, k, scale, VY_E4M3, 0, 0, 0, 0, group_size, pow2_shift(group_size),
                 reinterpret_cast<const __nv_bfloat16*>(x), x_stride, static_cast<int>(n_tokens),
                 reinterpret_cast<__nv_bfloat16*>(out), out_stride};
    return launch_gemv(1, p, as_stream(stream));
}
