// vy_decode_static.cu -- vy_moe_decode for callers that cannot allocate device memory.
//
// Some hosts of this library cannot call cudaMalloc: a language binding that is only ever handed
// tensor pointers by a runtime that owns all device memory, an engine whose memory planner has
// already given every byte away, or code that must not allocate at all while it runs (a stream
// under capture, a latency-critical loop).  They cannot provide vy_moe_decode's workspace, so this
// entry point takes its scratch from one array compiled into the library instead.
//
// The array lives in every GPU that loads the library and stays there until the process exits.
// Every call shares it and it keeps the previous call's contents; nothing in it needs to start at
// zero except the per-tile tickets of the down stage, which the routing-plan kernel of the same
// call clears before anything reads them.  Two calls whose kernels overlap on the GPU (different
// streams, or different host threads, without an ordering between them) race on the array and
// corrupt each other's results: order them on one stream.
#include <mutex>

#include "vy_moe.cuh"

namespace vy {
namespace {

static __device__ __align__(256) unsigned char g_decode_scratch[VY_DECODE_STATIC_SCRATCH_BYTES];

std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

// The device address of g_decode_scratch on the current device.  In host code the array's name
// is only a host-side stand-in, so the address comes from cudaGetSymbolAddress, once per device,
// with that device current (the first call on each device does this set-up).
int scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return fail(VY_ERR_CUDA, "vy_moe_decode_static: cudaGetDevice: %s", cudaGetErrorString(e));
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_scratch_addr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_decode_scratch);
        if (e != cudaSuccess || p == nullptr)
            return fail(VY_ERR_CUDA, "vy_moe_decode_static: cudaGetSymbolAddress: %s",
                        cudaGetErrorString(e));
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return VY_OK;
}

}  // namespace

int decode_static_scratch(void** out) { return scratch_address(out); }

}  // namespace vy

using namespace vy;

extern "C" int vy_moe_decode_static(const vy_moe_call* call, void* stream) {
    int st;
    if (!device_info(&st)) return st;
    if (!call || !call->geom) return fail(VY_ERR_INVALID, "vy_moe_decode_static: null call or geometry");
    vy_moe_call local = *call;
    size_t need = vy_moe_workspace_size(&local, 0);
    if (need > VY_DECODE_STATIC_SCRATCH_BYTES && local.k_splits == 0) {
        local.k_splits = 1;   // the split-K partials are what does not fit: run unsplit
        need = vy_moe_workspace_size(&local, 0);
    }
    if (need > VY_DECODE_STATIC_SCRATCH_BYTES)
        return fail(VY_ERR_UNSUPPORTED,
                    "vy_moe_decode_static: this call needs %zu bytes of scratch, more than the %zu "
                    "bytes built into the library (VY_DECODE_STATIC_SCRATCH_BYTES); pass a "
                    "workspace to vy_moe_decode instead",
                    need, static_cast<size_t>(VY_DECODE_STATIC_SCRATCH_BYTES));
    void* scratch = nullptr;
    if ((st = scratch_address(&scratch)) != VY_OK) return st;
    local.workspace = scratch;
    local.workspace_bytes = VY_DECODE_STATIC_SCRATCH_BYTES;
    return vy_moe_decode(&local, stream);
}
