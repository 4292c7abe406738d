"""vaayu_b200: archish9/Vaayu's fused packed-int4 MoE expert path, rebuilt for B200 (sm_100a).

The operator surface the engine's MoE patch calls, with the same names and semantics as the
reference (vaayu/packed_expert_kernels.py, vaayu/moe_patch.py's packed-expert helpers and the
DeepSeek-V4 block-scaled dequant), running on libvaayu_b200's CUDA kernels.  There is no CPU,
torch or Triton fallback: calls on CPU tensors or geometry the kernels do not take raise.
"""
from .arena import ExpertArena
from .block_scaled import (dequantize_block_scaled, dequantize_fp4_block_scaled, fp4_gemv,
                           fp8_gemv)
from .checkpoint import Checkpoint, group_packed_tensors_by_weight, packed_roles_complete
from .moe_patch import (accumulate_expert_outputs, build_expert_blob, compute_expert_dispatch,
                        dequantize_expert_blob, dequantize_expert_weights,
                        dequantize_packed_weight, expert_weights_from_entry, route_experts,
                        route_permute, topk_softmax, unpack_int32_to_int8)
from .packed_expert_kernels import (PATH_DECODE, PATH_PREFILL, ExpertTable, combine,
                                    install_packed_expert_kernels, moe_forward, moe_forward_with_shared,
                                    shared_expert_forward,
                                    moe_workspace_bytes, packed_experts_decode,
                                    packed_experts_decode_graphed, packed_experts_prefill)

__all__ = [
    "PATH_DECODE", "PATH_PREFILL", "Checkpoint", "ExpertArena", "ExpertTable", "accumulate_expert_outputs",
    "build_expert_blob", "combine", "compute_expert_dispatch", "dequantize_block_scaled",
    "dequantize_expert_blob", "dequantize_expert_weights", "dequantize_fp4_block_scaled",
    "dequantize_packed_weight", "expert_weights_from_entry", "fp4_gemv", "fp8_gemv",
    "group_packed_tensors_by_weight", "install_packed_expert_kernels", "moe_forward",
    "moe_forward_with_shared", "moe_workspace_bytes", "packed_roles_complete", "shared_expert_forward",
    "packed_experts_decode", "packed_experts_decode_graphed", "packed_experts_prefill",
    "route_experts", "route_permute", "topk_softmax", "unpack_int32_to_int8",
]
