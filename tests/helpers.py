"""Test helpers shared by the CPU and GPU suites: fixture loading, comparison metrics, and the
conversion between torch tensors and the oracle's numpy conventions (bf16 as uint16 bits)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
CODE = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}
NP16 = {0: np.uint16, 1: np.float16}


def golden(name: str):
    return np.load(GOLDEN / f"{name}.npz")


def geom(hid: int, inter: int, bits: int = 4, gs: int = 128):
    """The blob geometry tuple `build_expert_blob` derives: roles in gate, down, up order."""
    return (bits, gs, (("gate", inter, hid), ("down", hid, inter), ("up", inter, hid)))


def to_np(t: torch.Tensor) -> np.ndarray:
    """torch -> numpy in the oracle's convention (bf16 -> uint16 bits)."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype in (torch.float8_e4m3fn, torch.float8_e8m0fnu):
        return t.view(torch.uint8).numpy()
    return t.numpy()


def from_np(a: np.ndarray, code: int | None = None) -> torch.Tensor:
    """numpy -> torch; uint16 with code 0 (or None) is read as bf16 bits."""
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16 and code in (None, 0):
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
    if a.dtype == np.uint16 and code == 1:
        return torch.from_numpy(a.view(np.float16).copy())
    return torch.from_numpy(a.copy())


def f32(a: np.ndarray, code: int = 0) -> np.ndarray:
    """A bf16-bits / fp16 / fp32 array as float64 values."""
    if np.asarray(a).dtype == np.uint16 and code == 0:
        return (np.asarray(a).astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    return np.asarray(a).astype(np.float64)


def rel_l2(got, ref) -> float:
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))


def max_abs_over_rms(got, ref) -> float:
    """The north-star tolerance metric: max |got - ref| / RMS(ref); the bar is 2e-2."""
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    rms = float(np.sqrt(np.mean(ref * ref)))
    return float(np.max(np.abs(got - ref)) / max(rms, 1e-30))


def bf16_round_np(f) -> np.ndarray:
    """float values -> bf16 bits, round to nearest even."""
    f = np.asarray(f, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def expert_from_components(by_role: dict) -> dict:
    """Oracle expert dict (flat streams in gate, down, up order) from compressed-tensors
    components, the same concatenation `build_expert_blob` performs."""
    roles = ("gate", "down", "up")
    packed = np.concatenate([to_np(by_role[r]["weight_packed"]).reshape(-1) for r in roles])
    scale = np.concatenate([to_np(by_role[r]["weight_scale"]).reshape(-1) for r in roles])
    zero = None
    if "weight_zero_point" in by_role["gate"]:
        zero = np.concatenate([to_np(by_role[r]["weight_zero_point"]).reshape(-1) for r in roles])
    return {"packed": packed.astype(np.int32), "scale": scale, "zero": zero}
