// vy_common.cuh -- shared host and device helpers of libvaayu_b200 (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <utility>

#include "../../include/vaayu_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libvaayu_b200 is built for sm_100a only"
#endif

namespace vy {

// ── host: error plumbing ──────────────────────────────────────────────────────────────────

// Records the calling thread's last error and returns `code`.
int fail(int code, const char* fmt, ...);
// Clears the calling thread's last error; returns VY_OK.
int ok();
// VY_ERR_CUDA when a launch on this thread left an error, else VY_OK.
int check_launch(const char* what);
// Immutable per-device properties (filled once per device).
struct DeviceInfo {
    int sm_count;
    int major, minor;
    size_t smem_optin;
};
const DeviceInfo* device_info(int* status);
constexpr int kMaxDevices = 64;
// The current device's index, or -1 (with the error recorded) when the runtime cannot tell.
int current_device();
// Kernel attributes (shared-memory opt-in) and occupancy figures belong to one device: runs
// `setup` the first time (current device, key) succeeds, under a lock; later calls return VY_OK
// at once.  A failed setup is tried again on the next call.  Thread-safe.
int once_per_device(const void* key, int (*setup)(int device, void* ctx), void* ctx);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ── device: rounding to the activation dtype ─────────────────────────────────────────────

// fp32 value rounded (nearest even) to bf16 / fp16 and widened back; NaN passes through.
template <int ACT>
__device__ __forceinline__ float round_act(float v) {
    if constexpr (ACT == VY_BF16) {
        return __bfloat162float(__float2bfloat16_rn(v));
    } else if constexpr (ACT == VY_F16) {
        return __half2float(__float2half_rn(v));
    } else {
        return v;
    }
}

__device__ __forceinline__ float load_as_float(const void* p, int dtype, int64_t i) {
    switch (dtype) {
        case VY_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
        case VY_F16: return __half2float(reinterpret_cast<const __half*>(p)[i]);
        default: return reinterpret_cast<const float*>(p)[i];
    }
}

template <int SC>
__device__ __forceinline__ float load_scale(const void* p, int64_t i) {
    if constexpr (SC == VY_BF16) {
        return __bfloat162float(__ldg(reinterpret_cast<const __nv_bfloat16*>(p) + i));
    } else if constexpr (SC == VY_F16) {
        return __half2float(__ldg(reinterpret_cast<const __half*>(p) + i));
    } else {
        return __ldg(reinterpret_cast<const float*>(p) + i);
    }
}

// ── device: packed 16-bit pair arithmetic ────────────────────────────────────────────────

// (lo, hi) 16-bit patterns of one activation-dtype pair.
template <int ACT>
__device__ __forceinline__ uint32_t pair_sub(uint32_t a, uint32_t b) {
    uint32_t d;
    if constexpr (ACT == VY_BF16) {
        asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    } else {
        asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    }
    return d;
}

template <int ACT>
__device__ __forceinline__ uint32_t pair_mul(uint32_t a, uint32_t b) {
    uint32_t d;
    if constexpr (ACT == VY_BF16) {
        asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    } else {
        asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    }
    return d;
}

// The 16-bit pattern of `v` rounded to the activation dtype.
template <int ACT>
__device__ __forceinline__ uint32_t act_bits(float v) {
    if constexpr (ACT == VY_BF16) {
        return static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v)));
    } else {
        return static_cast<uint32_t>(__half_as_ushort(__float2half_rn(v)));
    }
}

template <int ACT>
__device__ __forceinline__ float act_from_bits(uint32_t b) {
    if constexpr (ACT == VY_BF16) {
        return __bfloat162float(__ushort_as_bfloat16(static_cast<unsigned short>(b)));
    } else {
        return __half2float(__ushort_as_half(static_cast<unsigned short>(b)));
    }
}

// Magic-number unpack of an int4 word: pair j (0..3) = (code j, code j+4) as activation-dtype
// values M + code, M = 128 (bf16: 0x4300 | c) or 1024 (fp16: 0x6400 | c).  Both are exact.
template <int ACT>
__device__ __forceinline__ uint32_t int4_pair(uint32_t word, int j) {
    constexpr uint32_t kMagic = (ACT == VY_BF16) ? 0x43004300u : 0x64006400u;
    return ((word >> (4 * j)) & 0x000F000Fu) | kMagic;
}

// M + z as a broadcast pair: the value the magic-number codes are reduced by.
template <int ACT>
__device__ __forceinline__ uint32_t int4_bias_pair(uint32_t z) {
    constexpr uint32_t kMagic = (ACT == VY_BF16) ? 0x4300u : 0x6400u;
    uint32_t v = kMagic | (z & 15u);
    return v | (v << 16);
}

// One byte of NVFP4 codes (two e2m1 values, low nibble first) as an exact f16 pair, by the
// hardware conversion.  One byte per asm statement: a form that unpacked a word into four byte
// registers in one statement produced wrong values for half of a fragment's rows in one kernel.
__device__ __forceinline__ uint32_t e2m1x2_f16(uint32_t byte) {
    uint32_t d;
    asm("{ .reg .b8 t;\n  cvt.u8.u32 t, %1;\n  cvt.rn.f16x2.e2m1x2 %0, t;\n}" : "=r"(d) : "r"(byte & 0xFFu));
    return d;
}

// ── device: tensor-core fragments (m16n8k16, fp32 accumulate) ────────────────────────────

template <int ACT>
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
    if constexpr (ACT == VY_BF16) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, "
            "{%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, "
            "{%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
}

// ── device: asynchronous copies ──────────────────────────────────────────────────────────

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint4 lds_v4(const void* smem) {
    uint4 v;
    uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(s));
    return v;
}

// Programmatic dependent launch: wait for the grid this one depends on / let dependents start.
__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dependents_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launch chained to the previous kernel on the stream (programmatic stream serialisation): the
// kernel must call grid_dependency_wait() before it touches memory.  Back-to-back launches then
// overlap the next kernel's launch with the previous one's tail.
template <typename... KArgs, typename... Args>
cudaError_t launch_chained(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                           Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Row-index permutation inside each 8-element group that lines activations up with the
// (code j, code j+4) pairs `int4_pair` produces: element k of a group sits at 2*(k%4) + k/4.
__host__ __device__ __forceinline__ int perm8(int k) { return ((k & 7) & 3) * 2 + ((k & 7) >> 2) + (k & ~7); }

}  // namespace vy
