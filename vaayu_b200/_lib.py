"""ctypes binding of libvaayu_b200.so (the C ABI declared in include/vaayu_b200.h).

The library is loaded on first use.  There is no fallback: if it is missing, or a call returns an
error status, a Python exception is raised -- NotImplementedError for geometry the kernels do not
take (VY_ERR_UNSUPPORTED), RuntimeError for everything else.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libvaayu_b200.so"

VY_OK, VY_ERR_UNSUPPORTED = 0, -1
BF16, F16, F32, E4M3, E8M0, I32, I64 = 0, 1, 2, 3, 4, 5, 6
DTYPE_CODE = {torch.bfloat16: BF16, torch.float16: F16, torch.float32: F32,
              torch.float8_e4m3fn: E4M3, torch.float8_e8m0fnu: E8M0, torch.int32: I32,
              torch.int64: I64}

P, I64T, I32T, SZ = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_size_t


class ExpertGeom(ctypes.Structure):
    """vy_expert_geom: role offsets index 0 gate, 1 up, 2 down."""
    _fields_ = [("hidden", I32T), ("inter", I32T), ("bits", I32T), ("group_size", I32T),
                ("scale_dtype", I32T), ("has_zero", I32T), ("word_off", I64T * 3),
                ("scale_off", I64T * 3), ("zero_off", I64T * 3)]


class MoeCall(ctypes.Structure):
    """vy_moe_call."""
    _fields_ = [("geom", ctypes.POINTER(ExpertGeom)), ("act_dtype", I32T), ("n_experts", I32T),
                ("top_k", I32T), ("ids_dtype", I32T), ("n_tokens", I64T), ("x", P),
                ("x_row_stride", I64T), ("expert_table", P), ("expert_ids", P), ("weights", P),
                ("w_dtype", I32T), ("reserved0", I32T), ("w_tok_stride", I64T),
                ("w_slot_stride", I64T), ("w_index", P), ("out", P), ("out_row_stride", I64T),
                ("contrib", P), ("h_out", P), ("workspace", P), ("workspace_bytes", SZ),
                ("stage_events", P), ("n_stage_events", I32T), ("reserved1", I32T),
                ("col_blocks", I32T), ("expert_base", I32T), ("ids_row_stride", I64T),
                ("shared_last", I32T), ("k_splits", I32T), ("result", P), ("result_row_stride", I64T)]


# name -> (restype, argtypes); every symbol include/vaayu_b200.h declares
SIGNATURES = {
    "vy_last_error": (ctypes.c_char_p, []),
    "vy_abi_version": (ctypes.c_int, []),
    "vy_unpack_int32_to_int8": (ctypes.c_int, [P, I64T, I64T, I32T, I64T, P, P]),
    "vy_dequant_flat": (ctypes.c_int, [P, I64T, I32T, P, I32T, I32T, P, I32T, P]),
    "vy_dequant_packed_weight": (ctypes.c_int, [P, I64T, I64T, I32T, P, I32T, I32T, P, P, I32T, P]),
    "vy_fp8_dequant": (ctypes.c_int, [P, I64T, I64T, P, I32T, I64T, I64T, P, I32T, P]),
    "vy_fp4_dequant": (ctypes.c_int, [P, I64T, I64T, P, I32T, P, I32T, P]),
    "vy_fp8_gemv": (ctypes.c_int, [P, I64T, I64T, P, I32T, I64T, I64T, P, I64T, I64T, P, I64T, P]),
    "vy_fp4_gemv": (ctypes.c_int, [P, I64T, I64T, P, I32T, P, I64T, I64T, P, I64T, P]),
    "vy_moe_topk_softmax": (ctypes.c_int, [P, I32T, I64T, I64T, I32T, I32T, P, P, P]),
    "vy_moe_route_permute": (ctypes.c_int, [P, I32T, I64T, I32T, I32T, P, P, P, P, P, P]),
    "vy_moe_workspace_size": (SZ, [ctypes.POINTER(MoeCall), I32T]),
    "vy_moe_decode": (ctypes.c_int, [ctypes.POINTER(MoeCall), P]),
    "vy_moe_decode_static": (ctypes.c_int, [ctypes.POINTER(MoeCall), P]),
    "vy_moe_prefill": (ctypes.c_int, [ctypes.POINTER(MoeCall), P]),
    "vy_moe_combine": (ctypes.c_int, [P, P, I32T, I64T, I32T, I64T, P, I64T, P]),
    "vy_sum_ordered": (ctypes.c_int, [P, I32T, I64T, P, P]),
    "vy_ep_dispatch_plan": (ctypes.c_int, [P, I32T, I64T, I64T, I32T, I32T, I32T, I32T, P, I32T, I64T, I64T,
                                           P, I32T, I64T, I64T, I64T, P, P, P, P, P, P, P]),
    "vy_ep_combine": (ctypes.c_int, [P, P, P, I32T, I64T, I64T, I32T, I64T, P, I64T, P]),
    "vy_moe_error_flags": (ctypes.c_int, [ctypes.POINTER(MoeCall), I32T, P, P]),
    "vy_selftest_bounded_wait": (ctypes.c_int, [I32T, I64T, P, P]),
}

_LIB = None
_LOCK = threading.Lock()


def lib() -> ctypes.CDLL:
    """The loaded library (loaded once).  Raises if it has not been built."""
    global _LIB
    if _LIB is None:
        with _LOCK:
            if _LIB is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(
                        f"{LIB_PATH.name} is not built; run `python -m vaayu_b200.build` "
                        "(vaayu_b200 has no CPU or Triton fallback)")
                handle = ctypes.CDLL(str(LIB_PATH))
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                _LIB = handle
    return _LIB


def check(status: int, what: str) -> None:
    if status == VY_OK:
        return
    msg = lib().vy_last_error().decode(errors="replace")
    if status == VY_ERR_UNSUPPORTED:
        raise NotImplementedError(f"{what}: {msg}")
    raise RuntimeError(f"{what} failed (status {status}): {msg}")


def ptr(t: "torch.Tensor | None") -> "int | None":
    return None if t is None else t.data_ptr()


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors, what: str) -> torch.device:
    """The common CUDA device of `tensors`; raises for CPU tensors or mixed devices.  Callers
    enqueue under `torch.cuda.device(dev)` so the launch lands on that device."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise RuntimeError(f"{what}: vaayu_b200 runs on CUDA tensors only (got {t.device})")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"{what}: tensors on {dev} and {t.device}")
    if dev is None:
        raise RuntimeError(f"{what}: no tensor argument")
    return dev
