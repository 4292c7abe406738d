// vy_capi.cu -- status plumbing and the per-device property cache of libvaayu_b200.
#include <map>
#include <mutex>
#include <utility>

#include "vy_common.cuh"

namespace vy {

namespace {
thread_local char g_last_error[512] = "";
DeviceInfo g_info[kMaxDevices];
bool g_have[kMaxDevices] = {};
std::mutex g_info_mu;
std::mutex g_once_mu;
std::map<std::pair<int, const void*>, int> g_once;   // (device, key) set up
}  // namespace

int current_device() {
    int dev = -1;
    const cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        fail(VY_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
        return -1;
    }
    return dev;
}

int once_per_device(const void* key, int (*setup)(int device, void* ctx), void* ctx) {
    const int dev = current_device();
    if (dev < 0) return VY_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_once_mu);
    if (g_once.count({dev, key})) return VY_OK;
    const int st = setup(dev, ctx);
    if (st == VY_OK) g_once[{dev, key}] = st;
    return st;
}

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

int ok() {
    g_last_error[0] = '\0';
    return VY_OK;
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(VY_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return ok();
}

const DeviceInfo* device_info(int* status) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        *status = fail(VY_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(g_info_mu);
    if (!g_have[dev]) {
        cudaDeviceProp p;
        e = cudaGetDeviceProperties(&p, dev);
        if (e != cudaSuccess) {
            *status = fail(VY_ERR_CUDA, "cudaGetDeviceProperties: %s", cudaGetErrorString(e));
            return nullptr;
        }
        g_info[dev] = DeviceInfo{p.multiProcessorCount, p.major, p.minor, p.sharedMemPerBlockOptin};
        g_have[dev] = true;
    }
    if (g_info[dev].major != 10 || g_info[dev].minor != 0) {
        *status = fail(VY_ERR_DEVICE, "device %d is sm_%d%d; libvaayu_b200 runs on sm_100 only", dev,
                       g_info[dev].major, g_info[dev].minor);
        return nullptr;
    }
    *status = VY_OK;
    return &g_info[dev];
}

}  // namespace vy

extern "C" const char* vy_last_error(void) { return vy::g_last_error; }

extern "C" int vy_abi_version(void) { return VY_ABI_VERSION; }
