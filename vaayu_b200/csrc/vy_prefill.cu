// vy_prefill.cu -- the tensor-core (tcgen05 / TMEM) grouped-GEMM expert layer for prefill.
#include "vy_moe.cuh"

namespace vy {
size_t prefill_workspace_bytes(const vy_moe_call* c) {
    (void)c;
    return 0;
}
}  // namespace vy

using namespace vy;

extern "C" int vy_moe_prefill(const vy_moe_call* c, void* stream) {
    (void)c;
    (void)stream;
    return fail(VY_ERR_UNSUPPORTED, "vy_moe_prefill: not built yet");
}
