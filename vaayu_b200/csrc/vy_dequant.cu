// vy_dequant.cu -- standalone dequant kernels: int-b packed (flat blob stream and one
// projection, with optional row-packed zero points), the int8 unpack, FP8-e4m3 block-scaled
// and FP4-e2m1 (NVFP4) dequant.  All are HBM-bound element-wise passes: each thread reads one
// 16-byte vector of codes where the layout allows it and writes the widened values with
// 16-byte stores; grids are a multiple of the SM count with a grid-stride loop.
#include <cuda_fp8.h>

#include "vy_common.cuh"

namespace vy {
namespace {

constexpr int kThreads = 256;

int grid_for(int64_t items, int sm_count) {
    int64_t blocks = (items + kThreads - 1) / kThreads;
    int64_t cap = static_cast<int64_t>(sm_count) * 8;
    if (blocks > cap) blocks = cap;
    return static_cast<int>(blocks < 1 ? 1 : blocks);
}

template <int OUT>
__device__ __forceinline__ void store_out(void* out, int64_t i, float v) {
    if constexpr (OUT == VY_BF16) {
        reinterpret_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
    } else if constexpr (OUT == VY_F16) {
        reinterpret_cast<__half*>(out)[i] = __float2half_rn(v);
    } else {
        reinterpret_cast<float*>(out)[i] = v;
    }
}

// ── int-b packed ──────────────────────────────────────────────────────────────────────────

// One word of codes -> `per` outputs at out[first ...].  w = act(act(u - z) * act(s)).
template <int ACT, int BITS>
__device__ __forceinline__ void dequant_word(uint32_t word, float s_act, float z, void* out,
                                             int64_t first, int64_t limit, bool vec_ok) {
    constexpr int kPer = 32 / BITS;
    constexpr uint32_t kMask = (1u << BITS) - 1u;
    float v[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        float code = static_cast<float>((word >> (BITS * j)) & kMask) - z;   // exact
        v[j] = round_act<ACT>(__fmul_rn(round_act<ACT>(code), s_act));
    }
    if constexpr (ACT != VY_F32 && kPer == 8) {
        if (vec_ok && first + kPer <= limit) {
            uint4 pk;
            uint32_t* q = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
            for (int j = 0; j < 4; ++j) q[j] = act_bits<ACT>(v[2 * j]) | (act_bits<ACT>(v[2 * j + 1]) << 16);
            *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + first) = pk;
            return;
        }
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j)
        if (first + j < limit) store_out<ACT>(out, first + j, v[j]);
}

template <int ACT, int SC, int BITS>
__global__ void __launch_bounds__(kThreads) dequant_flat_kernel(const int32_t* __restrict__ packed,
                                                                int64_t n_words, const void* scale,
                                                                int gs, void* out, bool vec_ok) {
    constexpr int kPer = 32 / BITS;
    const float off = static_cast<float>(1 << (BITS - 1));
    const int64_t limit = n_words * kPer;
    for (int64_t w = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; w < n_words;
         w += int64_t(gridDim.x) * blockDim.x) {
        uint32_t word = static_cast<uint32_t>(__ldg(packed + w));
        float s = round_act<ACT>(load_scale<SC>(scale, (w * kPer) / gs));
        dequant_word<ACT, BITS>(word, s, off, out, w * kPer, limit, vec_ok);
    }
}

template <int ACT, int SC, int BITS>
__global__ void __launch_bounds__(kThreads) dequant_role_kernel(
    const int32_t* __restrict__ packed, int64_t rows, int64_t cols, const void* scale, int gs,
    const int32_t* __restrict__ zero, void* out, bool vec_ok) {
    constexpr int kPer = 32 / BITS;
    const int64_t wpr = cols / kPer, groups = cols / gs, n_words = rows * wpr;
    const float off = static_cast<float>(1 << (BITS - 1));
    for (int64_t w = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; w < n_words;
         w += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = w / wpr, c0 = (w % wpr) * kPer, g = c0 / gs;
        uint32_t word = static_cast<uint32_t>(__ldg(packed + w));
        float s = round_act<ACT>(load_scale<SC>(scale, r * groups + g));
        float z = off;
        if (zero != nullptr) {
            uint32_t zw = static_cast<uint32_t>(__ldg(zero + (r / kPer) * groups + g));
            z = static_cast<float>((zw >> (BITS * (r % kPer))) & ((1u << BITS) - 1u));
        }
        dequant_word<ACT, BITS>(word, s, z, out, r * cols + c0, rows * cols, vec_ok);
    }
}

template <int BITS>
__global__ void __launch_bounds__(kThreads) unpack_kernel(const int32_t* __restrict__ packed,
                                                          int64_t rows, int64_t wpr, int64_t cols,
                                                          int8_t* __restrict__ out) {
    constexpr int kPer = 32 / BITS;
    const int64_t n_words = rows * wpr;
    for (int64_t w = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; w < n_words;
         w += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = w / wpr, c0 = (w % wpr) * kPer;
        uint32_t word = static_cast<uint32_t>(__ldg(packed + w));
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            if (c0 + j < cols) {
                int code = static_cast<int>((word >> (BITS * j)) & ((1u << BITS) - 1u));
                out[r * cols + c0 + j] = static_cast<int8_t>(code - (1 << (BITS - 1)));
            }
        }
    }
}

// ── FP8 / FP4 ─────────────────────────────────────────────────────────────────────────────

__device__ __forceinline__ float e4m3_to_float(uint8_t b) {
    __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(b), __NV_E4M3);
    return __half2float(__half(h));
}

__device__ __forceinline__ float e8m0_to_float(uint8_t b) {
    if (b == 0xFF) return __int_as_float(0x7FC00000);
    if (b == 0) return 5.877471754111438e-39f;   // 2^-127 (an fp32 subnormal)
    return __int_as_float(static_cast<int>(b) << 23);
}

template <int SC>
__device__ __forceinline__ float load_block_scale(const void* p, int64_t i) {
    if constexpr (SC == VY_E8M0) {
        return e8m0_to_float(__ldg(reinterpret_cast<const uint8_t*>(p) + i));
    } else {
        return load_scale<SC>(p, i);
    }
}

// e2m1 code (sign bit 3, exponent bits 1-2 with bias 1, mantissa bit 0) as a float.
__device__ __forceinline__ float e2m1_to_float(uint32_t nib) {
    uint32_t e = (nib >> 1) & 3u, m = nib & 1u;
    uint32_t bits = e ? (((e + 126u) << 23) | (m << 22)) : (m ? 0x3F000000u : 0u);
    return __uint_as_float(bits | ((nib & 8u) << 28));
}

template <int SC, int OUT>
__global__ void __launch_bounds__(kThreads) fp8_dequant_kernel(
    const uint8_t* __restrict__ w, int64_t rows, int64_t cols, const void* scale, int64_t scols,
    int64_t bo, int64_t bi, void* out, bool vec_ok) {
    const int64_t n = rows * cols, chunks = (n + 15) / 16;
    for (int64_t q = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; q < chunks;
         q += int64_t(gridDim.x) * blockDim.x) {
        const int64_t first = q * 16;
        uint8_t b[16];
        if (vec_ok && first + 16 <= n) {
            *reinterpret_cast<uint4*>(b) = __ldg(reinterpret_cast<const uint4*>(w + first));
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) b[j] = first + j < n ? w[first + j] : 0;
        }
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int64_t i = first + j, r = i / cols, c = i % cols;
            float s = load_block_scale<SC>(scale, (r / bo) * scols + c / bi);
            v[j] = __fmul_rn(e4m3_to_float(b[j]), s);
        }
        if constexpr (OUT != VY_F32) {
            if (vec_ok && first + 16 <= n) {
                uint4 pk[2];
                uint32_t* p32 = reinterpret_cast<uint32_t*>(pk);
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    p32[j] = act_bits<OUT>(v[2 * j]) | (act_bits<OUT>(v[2 * j + 1]) << 16);
                uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + first);
                dst[0] = pk[0];
                dst[1] = pk[1];
                continue;
            }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (first + j < n) store_out<OUT>(out, first + j, v[j]);
    }
}

template <int OUT>
__global__ void __launch_bounds__(kThreads) fp4_dequant_kernel(
    const uint8_t* __restrict__ w, int64_t rows, int64_t cols, const uint8_t* __restrict__ scale,
    int gs, void* out, bool vec_ok) {
    const int64_t n = rows * cols, chunks = (n + 15) / 16, groups = cols / gs;
    for (int64_t q = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; q < chunks;
         q += int64_t(gridDim.x) * blockDim.x) {
        const int64_t first = q * 16;
        uint8_t b[8];
        if (vec_ok && first + 16 <= n) {
            *reinterpret_cast<uint2*>(b) = __ldg(reinterpret_cast<const uint2*>(w + first / 2));
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) b[j] = first + 2 * j < n ? w[first / 2 + j] : 0;
        }
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int64_t i = first + j, r = i / cols, c = i % cols;
            float s = e4m3_to_float(__ldg(scale + r * groups + c / gs));
            uint32_t nib = (j & 1) ? (b[j >> 1] >> 4) : (b[j >> 1] & 15u);
            v[j] = __fmul_rn(e2m1_to_float(nib), s);
        }
        if constexpr (OUT != VY_F32) {
            if (vec_ok && first + 16 <= n) {
                uint4 pk[2];
                uint32_t* p32 = reinterpret_cast<uint32_t*>(pk);
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    p32[j] = act_bits<OUT>(v[2 * j]) | (act_bits<OUT>(v[2 * j + 1]) << 16);
                uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + first);
                dst[0] = pk[0];
                dst[1] = pk[1];
                continue;
            }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (first + j < n) store_out<OUT>(out, first + j, v[j]);
    }
}

// ── fast paths: whole 16-element chunks, each inside one row and one scale block ─────────────
//
// When the columns and the scale block width are multiples of 16, a chunk of 16 consecutive
// elements has one scale: the row / block arithmetic is done once per chunk (32-bit), the codes
// convert in pairs, and every thread keeps two chunks' loads in flight.  Same arithmetic as the
// element-wise kernels above: fp32 product of the exact decoded value and the scale (RN), then
// one rounding to the output dtype.

template <int OUT>
__device__ __forceinline__ void store16(void* out, uint32_t chunk, const float (&v)[16]) {
    if constexpr (OUT == VY_F32) {
        float4* d = reinterpret_cast<float4*>(out) + int64_t(chunk) * 4;
#pragma unroll
        for (int i = 0; i < 4; ++i) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
        uint32_t p32[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if constexpr (OUT == VY_BF16) {
                __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
                p32[j] = *reinterpret_cast<uint32_t*>(&h);
            } else {
                __half2 h = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
                p32[j] = *reinterpret_cast<uint32_t*>(&h);
            }
        }
        uint4* d = reinterpret_cast<uint4*>(out) + int64_t(chunk) * 2;
        d[0] = make_uint4(p32[0], p32[1], p32[2], p32[3]);
        d[1] = make_uint4(p32[4], p32[5], p32[6], p32[7]);
    }
}

// 16 e4m3 codes (one uint4) times one scale.
__device__ __forceinline__ void e4m3x16_times(const uint4 raw, float s, float (&v)[16]) {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const __nv_fp8x2_storage_t pr = static_cast<__nv_fp8x2_storage_t>((w[i] >> (16 * h)) & 0xFFFFu);
            const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(pr, __NV_E4M3);
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hr));
            v[4 * i + 2 * h] = __fmul_rn(f.x, s);
            v[4 * i + 2 * h + 1] = __fmul_rn(f.y, s);
        }
    }
}

template <int SC, int OUT>
__global__ void __launch_bounds__(kThreads) fp8_dequant_fast_kernel(const uint4* __restrict__ w, uint32_t chunks,
                                                                    uint32_t cpr, const void* scale, uint32_t scols,
                                                                    uint32_t bo, uint32_t bi16, void* out) {
    grid_dependency_wait();      // launched chained to the previous kernel on the stream
    grid_dependents_launch();
    const uint32_t stride = gridDim.x * blockDim.x;
    for (uint32_t q = blockIdx.x * blockDim.x + threadIdx.x; q < chunks; q += 2 * stride) {
        const uint32_t q2 = q + stride;
        const bool two = q2 < chunks;
        const uint4 a = __ldg(w + q);
        const uint4 b = two ? __ldg(w + q2) : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t ra = q / cpr, rb = q2 / cpr;
        const float sa = load_block_scale<SC>(scale, int64_t(ra / bo) * scols + (q - ra * cpr) / bi16);
        const float sb = two ? load_block_scale<SC>(scale, int64_t(rb / bo) * scols + (q2 - rb * cpr) / bi16) : 0.f;
        float v[16];
        e4m3x16_times(a, sa, v);
        store16<OUT>(out, q, v);
        if (two) {
            e4m3x16_times(b, sb, v);
            store16<OUT>(out, q2, v);
        }
    }
}

// 16 e2m1 codes (low nibble first) times one scale.  Each byte (two codes) goes to an f16 pair with
// the hardware conversion (exact: e2m1 values are 0, 0.5 .. 6), widened to fp32 (exact) and
// multiplied by the scale in fp32 -- the same product as decoding each code to fp32 directly.
__device__ __forceinline__ void e2m1x16_times(const uint2 raw, float s, float (&v)[16]) {
    const uint32_t w[2] = {raw.x, raw.y};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t h = e2m1x2_f16(w[i] >> (8 * j));
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
            v[8 * i + 2 * j] = __fmul_rn(f.x, s);
            v[8 * i + 2 * j + 1] = __fmul_rn(f.y, s);
        }
    }
}

template <int OUT>
__global__ void __launch_bounds__(kThreads) fp4_dequant_fast_kernel(const uint2* __restrict__ w, uint32_t chunks,
                                                                    uint32_t cpr, const uint8_t* __restrict__ scale,
                                                                    uint32_t groups, uint32_t gs16, void* out) {
    grid_dependency_wait();      // launched chained to the previous kernel on the stream
    grid_dependents_launch();
    const uint32_t stride = gridDim.x * blockDim.x;
    for (uint32_t q = blockIdx.x * blockDim.x + threadIdx.x; q < chunks; q += 2 * stride) {
        const uint32_t q2 = q + stride;
        const bool two = q2 < chunks;
        const uint2 a = __ldg(w + q);
        const uint2 b = two ? __ldg(w + q2) : make_uint2(0u, 0u);
        const uint32_t ra = q / cpr, rb = q2 / cpr;
        const float sa = e4m3_to_float(__ldg(scale + int64_t(ra) * groups + (q - ra * cpr) / gs16));
        const float sb = two ? e4m3_to_float(__ldg(scale + int64_t(rb) * groups + (q2 - rb * cpr) / gs16)) : 0.f;
        float v[16];
        e2m1x16_times(a, sa, v);
        store16<OUT>(out, q, v);
        if (two) {
            e2m1x16_times(b, sb, v);
            store16<OUT>(out, q2, v);
        }
    }
}

bool act_dtype_ok(int d) { return d == VY_BF16 || d == VY_F16 || d == VY_F32; }

// Dispatch (ACT x SC x BITS) for the two int-b kernels.
template <template <int, int, int> class Launch, typename... Args>
int dispatch_int(int act, int sc, int bits, Args... args) {
#define VY_CASE_BITS(A, S)                                             \
    switch (bits) {                                                    \
        case 2: return Launch<A, S, 2>::run(args...);                  \
        case 4: return Launch<A, S, 4>::run(args...);                  \
        case 8: return Launch<A, S, 8>::run(args...);                  \
        default: return fail(VY_ERR_UNSUPPORTED, "bits %d (2, 4, 8 supported)", bits); \
    }
#define VY_CASE_SC(A)                                                  \
    switch (sc) {                                                      \
        case VY_BF16: VY_CASE_BITS(A, VY_BF16)                         \
        case VY_F16: VY_CASE_BITS(A, VY_F16)                           \
        case VY_F32: VY_CASE_BITS(A, VY_F32)                           \
        default: return fail(VY_ERR_UNSUPPORTED, "scale dtype %d", sc); \
    }
    switch (act) {
        case VY_BF16: VY_CASE_SC(VY_BF16)
        case VY_F16: VY_CASE_SC(VY_F16)
        case VY_F32: VY_CASE_SC(VY_F32)
        default: return fail(VY_ERR_UNSUPPORTED, "output dtype %d", act);
    }
#undef VY_CASE_SC
#undef VY_CASE_BITS
}

struct FlatArgs {
    const int32_t* packed;
    int64_t n_words;
    const void* scale;
    int gs;
    void* out;
    bool vec_ok;
    int grid;
    cudaStream_t stream;
};

template <int A, int S, int B>
struct LaunchFlat {
    static int run(const FlatArgs& a) {
        dequant_flat_kernel<A, S, B><<<a.grid, kThreads, 0, a.stream>>>(a.packed, a.n_words, a.scale,
                                                                       a.gs, a.out, a.vec_ok);
        return check_launch("vy_dequant_flat");
    }
};

struct RoleArgs {
    const int32_t* packed;
    int64_t rows, cols;
    const void* scale;
    int gs;
    const int32_t* zero;
    void* out;
    bool vec_ok;
    int grid;
    cudaStream_t stream;
};

template <int A, int S, int B>
struct LaunchRole {
    static int run(const RoleArgs& a) {
        dequant_role_kernel<A, S, B><<<a.grid, kThreads, 0, a.stream>>>(
            a.packed, a.rows, a.cols, a.scale, a.gs, a.zero, a.out, a.vec_ok);
        return check_launch("vy_dequant_packed_weight");
    }
};

}  // namespace
}  // namespace vy

using namespace vy;

extern "C" int vy_unpack_int32_to_int8(const int32_t* packed, int64_t rows, int64_t words_per_row,
                                       int32_t bits, int64_t cols, int8_t* out, void* stream) {
    int st;
    const DeviceInfo* dev = device_info(&st);
    if (!dev) return st;
    if (rows < 0 || cols < 0 || words_per_row < 0) return fail(VY_ERR_INVALID, "negative size");
    if (bits != 2 && bits != 4 && bits != 8) return fail(VY_ERR_UNSUPPORTED, "bits %d", bits);
    if (words_per_row * (32 / bits) < cols) return fail(VY_ERR_INVALID, "too few words for cols");
    if (rows == 0 || words_per_row == 0) return ok();
    if (!packed || !out) return fail(VY_ERR_INVALID, "null pointer");
    int grid = grid_for(rows * words_per_row, dev->sm_count);
    cudaStream_t s = as_stream(stream);
    if (bits == 2) unpack_kernel<2><<<grid, kThreads, 0, s>>>(packed, rows, words_per_row, cols, out);
    if (bits == 4) unpack_kernel<4><<<grid, kThreads, 0, s>>>(packed, rows, words_per_row, cols, out);
    if (bits == 8) unpack_kernel<8><<<grid, kThreads, 0, s>>>(packed, rows, words_per_row, cols, out);
    return check_launch("vy_unpack_int32_to_int8");
}

extern "C" int vy_dequant_flat(const int32_t* packed, int64_t n_words, int32_t bits,
                               const void* scale, int32_t scale_dtype, int32_t group_size,
                               void* out, int32_t out_dtype, void* stream) {
    int st;
    const DeviceInfo* dev = device_info(&st);
    if (!dev) return st;
    if (n_words < 0) return fail(VY_ERR_INVALID, "negative size");
    if (bits != 2 && bits != 4 && bits != 8) return fail(VY_ERR_UNSUPPORTED, "bits %d", bits);
    if (group_size <= 0 || group_size % (32 / bits))
        return fail(VY_ERR_UNSUPPORTED, "group size %d does not hold whole %d-bit words", group_size, bits);
    if (!act_dtype_ok(out_dtype)) return fail(VY_ERR_UNSUPPORTED, "output dtype %d", out_dtype);
    if (n_words == 0) return ok();
    if (!packed || !scale || !out) return fail(VY_ERR_INVALID, "null pointer");
    FlatArgs a{packed, n_words, scale, group_size, out, aligned16(out),
               grid_for(n_words, dev->sm_count), as_stream(stream)};
    return dispatch_int<LaunchFlat>(out_dtype, scale_dtype, bits, a);
}

extern "C" int vy_dequant_packed_weight(const int32_t* packed, int64_t rows, int64_t cols,
                                        int32_t bits, const void* scale, int32_t scale_dtype,
                                        int32_t group_size, const int32_t* zero, void* out,
                                        int32_t out_dtype, void* stream) {
    int st;
    const DeviceInfo* dev = device_info(&st);
    if (!dev) return st;
    if (rows < 0 || cols < 0) return fail(VY_ERR_INVALID, "negative size");
    if (bits != 2 && bits != 4 && bits != 8) return fail(VY_ERR_UNSUPPORTED, "bits %d", bits);
    if (group_size <= 0 || group_size % (32 / bits) || cols % group_size)
        return fail(VY_ERR_UNSUPPORTED, "group size %d with %lld columns at %d bits", group_size,
                    static_cast<long long>(cols), bits);
    if (!act_dtype_ok(out_dtype)) return fail(VY_ERR_UNSUPPORTED, "output dtype %d", out_dtype);
    if (rows == 0 || cols == 0) return ok();
    if (!packed || !scale || !out) return fail(VY_ERR_INVALID, "null pointer");
    const int64_t per = 32 / bits;
    RoleArgs a{packed, rows, cols, scale, group_size, zero, out,
               aligned16(out) && (cols % 8 == 0), grid_for(rows * (cols / per), dev->sm_count),
               as_stream(stream)};
    return dispatch_int<LaunchRole>(out_dtype, scale_dtype, bits, a);
}

extern "C" int vy_fp8_dequant(const uint8_t* w, int64_t rows, int64_t cols, const void* scale,
                              int32_t scale_dtype, int64_t srows, int64_t scols, void* out,
                              int32_t out_dtype, void* stream) {
    int st;
    const DeviceInfo* dev = device_info(&st);
    if (!dev) return st;
    if (rows < 0 || cols < 0) return fail(VY_ERR_INVALID, "negative size");
    if (srows <= 0 || scols <= 0 || rows % srows || cols % scols)
        return fail(VY_ERR_INVALID, "scale [%lld, %lld] does not tile weight [%lld, %lld]",
                    (long long)srows, (long long)scols, (long long)rows, (long long)cols);
    if (!act_dtype_ok(out_dtype)) return fail(VY_ERR_UNSUPPORTED, "output dtype %d", out_dtype);
    if (rows == 0 || cols == 0) return ok();
    if (!w || !scale || !out) return fail(VY_ERR_INVALID, "null pointer");
    const bool vec = aligned16(w) && aligned16(out);
    const int grid = grid_for((rows * cols + 15) / 16, dev->sm_count);
    cudaStream_t s = as_stream(stream);
    const int64_t bo = rows / srows, bi = cols / scols;
    if (vec && cols % 16 == 0 && bi % 16 == 0 && rows * cols / 16 < (int64_t(1) << 31)) {
        const uint32_t chunks = static_cast<uint32_t>(rows * cols / 16), cpr = static_cast<uint32_t>(cols / 16);
        const int fgrid = grid_for((chunks + 1) / 2, dev->sm_count);
        const uint4* w4 = reinterpret_cast<const uint4*>(w);
        const uint32_t sc32 = static_cast<uint32_t>(scols), bo32 = static_cast<uint32_t>(bo),
                       b16 = static_cast<uint32_t>(bi / 16);
        cudaError_t e = cudaSuccess;
#define VY_FP8F(S, O) e = launch_chained(fp8_dequant_fast_kernel<S, O>, dim3(fgrid), dim3(kThreads), 0, s, w4, chunks, cpr, \
                                       scale, sc32, bo32, b16, out)
#define VY_FP8F_OUT(S)                                                  \
    switch (out_dtype) {                                                \
        case VY_BF16: VY_FP8F(S, VY_BF16); break;                       \
        case VY_F16: VY_FP8F(S, VY_F16); break;                         \
        default: VY_FP8F(S, VY_F32); break;                             \
    }
        switch (scale_dtype) {
            case VY_F32: VY_FP8F_OUT(VY_F32) break;
            case VY_BF16: VY_FP8F_OUT(VY_BF16) break;
            case VY_F16: VY_FP8F_OUT(VY_F16) break;
            case VY_E8M0: VY_FP8F_OUT(VY_E8M0) break;
            default: return fail(VY_ERR_UNSUPPORTED, "block-scale dtype %d", scale_dtype);
        }
#undef VY_FP8F_OUT
#undef VY_FP8F
        if (e != cudaSuccess) return fail(VY_ERR_CUDA, "vy_fp8_dequant launch: %s", cudaGetErrorString(e));
        return check_launch("vy_fp8_dequant");
    }
#define VY_FP8(S, O) fp8_dequant_kernel<S, O><<<grid, kThreads, 0, s>>>(w, rows, cols, scale, scols, bo, bi, out, vec)
#define VY_FP8_OUT(S)                                                   \
    switch (out_dtype) {                                                \
        case VY_BF16: VY_FP8(S, VY_BF16); break;                        \
        case VY_F16: VY_FP8(S, VY_F16); break;                          \
        default: VY_FP8(S, VY_F32); break;                              \
    }
    switch (scale_dtype) {
        case VY_F32: VY_FP8_OUT(VY_F32) break;
        case VY_BF16: VY_FP8_OUT(VY_BF16) break;
        case VY_F16: VY_FP8_OUT(VY_F16) break;
        case VY_E8M0: VY_FP8_OUT(VY_E8M0) break;
        default: return fail(VY_ERR_UNSUPPORTED, "block-scale dtype %d", scale_dtype);
    }
#undef VY_FP8_OUT
#undef VY_FP8
    return check_launch("vy_fp8_dequant");
}

extern "C" int vy_fp4_dequant(const uint8_t* w, int64_t rows, int64_t cols, const uint8_t* scale,
                              int32_t group_size, void* out, int32_t out_dtype, void* stream) {
    int st;
    const DeviceInfo* dev = device_info(&st);
    if (!dev) return st;
    if (rows < 0 || cols < 0) return fail(VY_ERR_INVALID, "negative size");
    if (cols % 2 || group_size <= 0 || cols % group_size)
        return fail(VY_ERR_INVALID, "columns %lld / group %d", (long long)cols, group_size);
    if (!act_dtype_ok(out_dtype)) return fail(VY_ERR_UNSUPPORTED, "output dtype %d", out_dtype);
    if (rows == 0 || cols == 0) return ok();
    if (!w || !scale || !out) return fail(VY_ERR_INVALID, "null pointer");
    const bool vec = (reinterpret_cast<uintptr_t>(w) & 7u) == 0 && aligned16(out);
    const int grid = grid_for((rows * cols + 15) / 16, dev->sm_count);
    cudaStream_t s = as_stream(stream);
    if (vec && cols % 16 == 0 && group_size % 16 == 0 && rows * cols / 16 < (int64_t(1) << 31)) {
        const uint32_t chunks = static_cast<uint32_t>(rows * cols / 16), cpr = static_cast<uint32_t>(cols / 16);
        const uint32_t groups = static_cast<uint32_t>(cols / group_size), g16 = static_cast<uint32_t>(group_size / 16);
        const int fgrid = grid_for((chunks + 1) / 2, dev->sm_count);
        const uint2* w2 = reinterpret_cast<const uint2*>(w);
        cudaError_t e;
        switch (out_dtype) {
            case VY_BF16: e = launch_chained(fp4_dequant_fast_kernel<VY_BF16>, dim3(fgrid), dim3(kThreads), 0, s, w2,
                                             chunks, cpr, scale, groups, g16, out); break;
            case VY_F16: e = launch_chained(fp4_dequant_fast_kernel<VY_F16>, dim3(fgrid), dim3(kThreads), 0, s, w2,
                                            chunks, cpr, scale, groups, g16, out); break;
            default: e = launch_chained(fp4_dequant_fast_kernel<VY_F32>, dim3(fgrid), dim3(kThreads), 0, s, w2,
                                        chunks, cpr, scale, groups, g16, out); break;
        }
        if (e != cudaSuccess) return fail(VY_ERR_CUDA, "vy_fp4_dequant launch: %s", cudaGetErrorString(e));
        return check_launch("vy_fp4_dequant");
    }
    switch (out_dtype) {
        case VY_BF16: fp4_dequant_kernel<VY_BF16><<<grid, kThreads, 0, s>>>(w, rows, cols, scale, group_size, out, vec); break;
        case VY_F16: fp4_dequant_kernel<VY_F16><<<grid, kThreads, 0, s>>>(w, rows, cols, scale, group_size, out, vec); break;
        default: fp4_dequant_kernel<VY_F32><<<grid, kThreads, 0, s>>>(w, rows, cols, scale, group_size, out, vec); break;
    }
    return check_launch("vy_fp4_dequant");
}
