"""Seeded synthetic pack-quantized MoE layers with the benchmark shapes.

The value distributions are the ones the benchmark configurations name: int4 codes uniform in
[0, 15], packed 8 per int32 along K (element j of a word at bits 4j, compressed-tensors'
`pack_to_int32` order); fp16 scales ~U(0.005, 0.02), one per `group` elements of a row; optional
int4 zero points uniform in [0, 15], packed along rows as compressed-tensors packs them
(`pack_to_int32(zp, bits, packed_dim=0)`); activations ~N(0, 1) in bf16; router logits ~N(0, 1),
softmax -> top-k -> renormalised (vaayu/moe_patch.py:160-161, 2331-2334).

Generator call order: for every expert the roles gate [I, H], down [H, I], up [I, H] (codes then
scales, then zero points when asked for); then the activations; then the router logits.  Works on
any device the generator lives on.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

GROUP = 128


def pack_codes(u: torch.Tensor, bits: int = 4) -> torch.Tensor:
    """[rows, cols] unsigned codes -> [rows, cols * bits / 32] int32 words."""
    per = 32 // bits
    rows, cols = u.shape
    u = u.to(torch.int32).reshape(rows, cols // per, per)
    p = torch.zeros(rows, cols // per, dtype=torch.int32, device=u.device)
    for j in range(per):
        p |= u[:, :, j] << (bits * j)
    return p


def pack_zero_points(z: torch.Tensor, bits: int = 4) -> torch.Tensor:
    """[rows, groups] unsigned zero codes -> [ceil(rows * bits / 32), groups] int32, packed along rows."""
    per = 32 // bits
    pad = (-z.shape[0]) % per
    if pad:
        z = F.pad(z, (0, 0, 0, pad))
    return pack_codes(z.t().contiguous(), bits).t().contiguous()


def make_role(rows: int, cols: int, gen: torch.Generator, group: int = GROUP, zeros: bool = False,
              scale_dtype: torch.dtype = torch.float16) -> dict:
    """One projection's compressed-tensors components: weight_packed / weight_scale / weight_shape
    (+ weight_zero_point)."""
    dev = gen.device
    u = torch.randint(0, 16, (rows, cols), dtype=torch.int32, generator=gen, device=dev)
    comps = {
        "weight_packed": pack_codes(u),
        "weight_scale": (torch.rand(rows, cols // group, generator=gen, device=dev) * 0.015
                         + 0.005).to(scale_dtype),
        "weight_shape": torch.tensor([rows, cols]),
    }
    if zeros:
        z = torch.randint(0, 16, (rows, cols // group), dtype=torch.int32, generator=gen, device=dev)
        comps["weight_zero_point"] = pack_zero_points(z)
    return comps


def make_expert(hidden: int, inter: int, gen: torch.Generator, group: int = GROUP,
                zeros: bool = False, scale_dtype: torch.dtype = torch.float16) -> dict:
    """{role: components} for one expert, roles drawn in gate, down, up order."""
    return {"gate": make_role(inter, hidden, gen, group, zeros, scale_dtype),
            "down": make_role(hidden, inter, gen, group, zeros, scale_dtype),
            "up": make_role(inter, hidden, gen, group, zeros, scale_dtype)}


def make_tokens(tokens: int, hidden: int, experts: int, top_k: int, gen: torch.Generator,
                skew: float = 0.0):
    """(x [T, H] bf16, routing weights [T, K] fp32, expert ids [T, K] int64): softmax top-k over
    N(0,1) logits, renormalised; `skew` adds linspace(0, skew, E) to the logits so expert loads
    differ (the prefill configuration's 4x spread)."""
    dev = gen.device
    x = torch.randn(tokens, hidden, generator=gen, device=dev).to(torch.bfloat16)
    logits = torch.randn(tokens, experts, generator=gen, device=dev)
    if skew:
        logits = logits + torch.linspace(0.0, skew, experts, device=dev)
    w, idx = torch.topk(logits.softmax(-1), top_k, -1)
    return x, w / w.sum(-1, keepdim=True), idx
