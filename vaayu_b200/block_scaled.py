"""Block-scaled FP8-e4m3 / FP4-e2m1 dequant (and dequant fused into a decode GEMV) on B200.

    dequantize_block_scaled(weight, scale, dtype=bf16)
        vaayu/model_code/deepseek_v4/modeling_deepseek_v4.py:228-240: `scale[i, j]` covers the
        tile weight[i*bo:(i+1)*bo, j*bi:(j+1)*bi], block sizes derived from the two shapes;
        out = dtype(float(w) * float(scale)).  e4m3 weights; fp32 / bf16 / fp16 / e8m0 scales.
    dequantize_fp4_block_scaled(weight_u8, scale_e4m3, dtype=bf16)
        NVFP4: two e2m1 codes per byte (low nibble = even column), one e4m3 scale per 16
        elements (group derived from the shapes).  No reference function exists; the e2m1 value
        set is the OCP MX one.  A `float4_e2m1fn_x2` tensor is read through a uint8 view.
    fp8_gemv / fp4_gemv
        y[t, n] = bf16(sum_k deq(W)[n, k] * x[t, k]) with fp32 accumulation, batch <= 16.
"""
from __future__ import annotations

import torch

from . import _lib


def _u8(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.uint8 else t.view(torch.uint8)


def dequantize_block_scaled(weight: torch.Tensor, scale: torch.Tensor,
                            dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    dev = _lib.require_cuda(weight, scale, what="dequantize_block_scaled")
    if weight.dtype != torch.float8_e4m3fn:
        raise NotImplementedError(f"block-scaled weight dtype {weight.dtype} (float8_e4m3fn)")
    sc = _lib.DTYPE_CODE.get(scale.dtype)
    if sc not in (_lib.F32, _lib.BF16, _lib.F16, _lib.E8M0):
        raise NotImplementedError(f"block-scale dtype {scale.dtype}")
    oc = _lib.DTYPE_CODE.get(dtype)
    if oc not in (_lib.BF16, _lib.F16, _lib.F32):
        raise NotImplementedError(f"output dtype {dtype}")
    w = weight.contiguous()
    s = scale.contiguous()
    rows, cols = w.shape
    out = torch.empty(rows, cols, dtype=dtype, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().vy_fp8_dequant(w.data_ptr(), rows, cols, s.data_ptr(), sc,
                                             s.shape[0], s.shape[1], out.data_ptr(), oc,
                                             _lib.stream_of(dev)), "dequantize_block_scaled")
    return out


def dequantize_fp4_block_scaled(weight_u8: torch.Tensor, scale_e4m3: torch.Tensor,
                                dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    dev = _lib.require_cuda(weight_u8, scale_e4m3, what="dequantize_fp4_block_scaled")
    w = _u8(weight_u8).contiguous()
    s = _u8(scale_e4m3).contiguous()
    rows, cols = w.shape[0], w.shape[1] * 2
    if s.shape[0] != rows or cols % s.shape[1]:
        raise ValueError(f"scale {tuple(s.shape)} does not tile fp4 weight [{rows}, {cols}]")
    oc = _lib.DTYPE_CODE.get(dtype)
    if oc not in (_lib.BF16, _lib.F16, _lib.F32):
        raise NotImplementedError(f"output dtype {dtype}")
    out = torch.empty(rows, cols, dtype=dtype, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().vy_fp4_dequant(w.data_ptr(), rows, cols, s.data_ptr(),
                                             cols // s.shape[1], out.data_ptr(), oc,
                                             _lib.stream_of(dev)), "dequantize_fp4_block_scaled")
    return out


def fp8_gemv(x: torch.Tensor, weight: torch.Tensor, scale: torch.Tensor,
             out: "torch.Tensor | None" = None) -> torch.Tensor:
    """x [T, K] bf16 (T <= 16) times the dequantised e4m3 weight [N, K] -> [T, N] bf16."""
    dev = _lib.require_cuda(x, weight, scale, out, what="fp8_gemv")
    if x.dtype != torch.bfloat16 or x.stride(-1) != 1:
        raise NotImplementedError("fp8_gemv: x must be bf16 with a unit last stride")
    w = weight.contiguous()
    s = scale.contiguous()
    sc = _lib.DTYPE_CODE.get(s.dtype)
    n, k = w.shape
    t = x.shape[0]
    if out is None:
        out = torch.empty(t, n, dtype=torch.bfloat16, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().vy_fp8_gemv(_u8(w).data_ptr(), n, k, s.data_ptr(), sc, s.shape[0],
                                          s.shape[1], x.data_ptr(), x.stride(0), t,
                                          out.data_ptr(), out.stride(0), _lib.stream_of(dev)),
                   "fp8_gemv")
    return out


def fp4_gemv(x: torch.Tensor, weight_u8: torch.Tensor, scale_e4m3: torch.Tensor,
             out: "torch.Tensor | None" = None) -> torch.Tensor:
    """x [T, K] bf16 (T <= 16) times the dequantised NVFP4 weight [N, K] -> [T, N] bf16."""
    dev = _lib.require_cuda(x, weight_u8, scale_e4m3, out, what="fp4_gemv")
    if x.dtype != torch.bfloat16 or x.stride(-1) != 1:
        raise NotImplementedError("fp4_gemv: x must be bf16 with a unit last stride")
    w = _u8(weight_u8).contiguous()
    s = _u8(scale_e4m3).contiguous()
    n, k = w.shape[0], w.shape[1] * 2
    t = x.shape[0]
    if out is None:
        out = torch.empty(t, n, dtype=torch.bfloat16, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().vy_fp4_gemv(w.data_ptr(), n, k, s.data_ptr(), k // s.shape[1],
                                          x.data_ptr(), x.stride(0), t, out.data_ptr(),
                                          out.stride(0), _lib.stream_of(dev)), "fp4_gemv")
    return out
