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


# ── GPU-suite helpers: the oracle on the same tensors the kernels see ─────────────────────

def oracle_expert(blob: dict) -> dict:
    """A `build_expert_blob` blob (any device) as the oracle's numpy expert dict."""
    f = blob["flat"]
    return {"packed": to_np(f["packed"]).astype(np.int32), "scale": to_np(f["scale"]),
            "zero": None if "zero" not in f else to_np(f["zero"]).astype(np.int32)}


def oracle_layer(blobs, x, eidx, rw, w_index=None, want_h=False, want_y=False, threads=0,
                 h_in=None):
    """Oracle of one layer call: blobs indexed by expert id; eidx [T, K]; rw [T, K] (or flat
    with w_index)."""
    from oracle import oracle as O
    experts = [oracle_expert(b) for b in blobs]
    sc = CODE[blobs[0]["flat"]["scale"].dtype]
    res = O.moe_layer(blobs[0]["geom"], experts, to_np(x), CODE[x.dtype], to_np(eidx),
                      to_np(rw.reshape(-1)) if w_index is None else to_np(rw.reshape(-1)),
                      CODE[rw.dtype], sc,
                      w_index=None if w_index is None else np.asarray(w_index, np.int32),
                      want_h=want_h, want_y=want_y, threads=threads, h_in=h_in)
    return res


def make_blobs(hid, inter, n, gs=128, seed=0, zeros=False, scale_dtype=None, device="cuda"):
    """n synthetic expert blobs (CPU generator, so every machine draws the same bits)."""
    import vaayu_b200 as vb
    from vaayu_b200 import synthetic
    scale_dtype = scale_dtype or torch.float16
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        by_role = synthetic.make_expert(hid, inter, g, group=gs, zeros=zeros, scale_dtype=scale_dtype)
        by_role = {r: {k: (v if k == "weight_shape" else v.to(device)) for k, v in c.items()}
                   for r, c in by_role.items()}
        out.append(vb.build_expert_blob(by_role))
    return out


def fp64_layer(blobs, x, eidx, rw):
    """The truth: the exact dequantised weights, float64 everywhere."""
    from oracle import oracle as O
    geom = blobs[0]["geom"]
    bits, gs, roles = geom
    lay = O.layout(geom)
    xf = f32(to_np(x), CODE[x.dtype])
    eidx = np.asarray(to_np(eidx)).reshape(xf.shape[0], -1)
    w = f32(to_np(rw), CODE[rw.dtype]).reshape(eidx.shape)
    out = np.zeros((xf.shape[0], lay["gate"][3]))
    mats_cache = {}
    for t in range(eidx.shape[0]):
        for k in range(eidx.shape[1]):
            e = int(eidx[t, k])
            if e not in mats_cache:
                ex = oracle_expert(blobs[e])
                mats = {}
                for role, rows, cols in roles:
                    w_at, s_at, _r, _c = lay[role]
                    es = ex["scale"]
                    d = O.dequant_role(ex["packed"][w_at:], rows, cols, bits, es[s_at:],
                                       CODE[blobs[e]["flat"]["scale"].dtype], gs, 2)
                    mats[role] = d.astype(np.float64)
                mats_cache[e] = mats
            m = mats_cache[e]
            g, u = m["gate"] @ xf[t], m["up"] @ xf[t]
            out[t] += (m["down"] @ (g / (1 + np.exp(-g)) * u)) * w[t, k]
    return out
