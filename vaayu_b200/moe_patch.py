"""The packed-expert helpers of archish9/Vaayu's MoE patch, on the B200 kernels.

Same names, arguments and error behaviour as vaayu/moe_patch.py's helpers for this path; the
arithmetic runs in libvaayu_b200 (CUDA, sm_100a).  CPU tensors are refused: there is no CPU
path behind these functions.

    unpack_int32_to_int8        vaayu/moe_patch.py:668-710
    dequantize_packed_weight    vaayu/moe_patch.py:713-744   (+ zero points, an extension)
    build_expert_blob           vaayu/moe_patch.py:794-846   (+ zero points, an extension)
    dequantize_expert_blob      vaayu/moe_patch.py:849-864
    expert_weights_from_entry   vaayu/moe_patch.py:867-877
    dequantize_expert_weights   vaayu/moe_patch.py:880-891
    accumulate_expert_outputs   vaayu/moe_patch.py:914-940
    route_experts               vaayu/moe_patch.py:130-167
    compute_expert_dispatch     vaayu/moe_patch.py:306-326

Zero points: the reference refuses `weight_zero_point` (NotImplementedError, :724-729, :811-818).
This build decodes them as w = act(act(u - z) * act(scale)), z the stored code of compressed-
tensors' row-packed zero points; z = 2^(b-1) everywhere is exactly the reference's symmetric
format.  Act-order `weight_g_idx` is still refused by name.
"""
from __future__ import annotations

import torch

from . import _lib

_ROLES = ("gate", "down", "up")


def _refuse_g_idx(comps: dict) -> None:
    if "weight_g_idx" in comps:
        raise NotImplementedError(
            "act-order pack-quantized experts carry a g_idx column permutation that vaayu_b200 "
            "does not apply; this checkpoint would decode to permuted weights. Supported: "
            "group quantization, symmetric or with zero points.")


def _scale_code(scale: torch.Tensor) -> int:
    code = _lib.DTYPE_CODE.get(scale.dtype)
    if code not in (_lib.BF16, _lib.F16, _lib.F32):
        raise NotImplementedError(f"scale dtype {scale.dtype}")
    return code


def _act_code(dtype: torch.dtype) -> int:
    code = _lib.DTYPE_CODE.get(dtype)
    if code not in (_lib.BF16, _lib.F16, _lib.F32):
        raise NotImplementedError(f"dequant output dtype {dtype}")
    return code


def unpack_int32_to_int8(packed: torch.Tensor, num_bits: int, cols: int) -> torch.Tensor:
    """Inverse of compressed-tensors' `pack_to_int32` along the last dim: element j of a word
    at bits [b*j, b*j+b), returned as the signed code (u - 2^(b-1)) in int8."""
    dev = _lib.require_cuda(packed, what="unpack_int32_to_int8")
    if 32 % num_bits:
        raise NotImplementedError(f"{num_bits}-bit codes straddle int32 words")
    packed = packed.contiguous()
    rows, words = packed.shape
    out = torch.empty(rows, cols, dtype=torch.int8, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().vy_unpack_int32_to_int8(
            packed.data_ptr(), rows, words, num_bits, cols, out.data_ptr(), _lib.stream_of(dev)),
            "unpack_int32_to_int8")
    return out


def dequantize_packed_weight(components: dict, dtype: torch.dtype) -> torch.Tensor:
    """One expert linear's dense weight from its pack-quantized components.  Bit width and group
    size are derived from the tensors (packed vs original element count; the scale's last dim)."""
    packed = components["weight_packed"]
    scale = components["weight_scale"]
    _refuse_g_idx(components)
    rows, cols = (int(x) for x in components["weight_shape"].tolist())
    num_bits, remainder = divmod(packed.numel() * 32, rows * cols)
    if remainder or not 1 <= num_bits <= 8:
        raise ValueError(f"cannot derive bit width: {packed.numel()} int32 words for a "
                         f"{rows}x{cols} weight")
    zero = components.get("weight_zero_point")
    dev = _lib.require_cuda(packed, scale, zero, what="dequantize_packed_weight")
    groups = scale.shape[-1]
    packed, scale = packed.contiguous(), scale.contiguous()
    zero = None if zero is None else zero.contiguous()
    out = torch.empty(rows, cols, dtype=dtype, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().vy_dequant_packed_weight(
            packed.data_ptr(), rows, cols, num_bits, scale.data_ptr(), _scale_code(scale),
            cols // groups, _lib.ptr(zero), out.data_ptr(), _act_code(dtype),
            _lib.stream_of(dev)), "dequantize_packed_weight")
    return out


def build_expert_blob(by_role: dict) -> "dict | None":
    """One expert's pack-quantized tensors as a single blob, or None when it cannot be decoded
    in one fused pass (a dense expert; roles at different bit widths or group sizes).

    {"flat": {"packed": int32 1-D, "scale": 1-D [, "zero": int32 1-D]},
     "geom": (bits, group, ((role, rows, cols), ...))} with roles in `by_role`'s order."""
    geom = []
    for role, comps in by_role.items():
        _refuse_g_idx(comps)
        if not {"weight_packed", "weight_scale", "weight_shape"} <= set(comps):
            return None
        rows, cols = (int(x) for x in comps["weight_shape"].tolist())
        num_bits, remainder = divmod(comps["weight_packed"].numel() * 32, rows * cols)
        geom.append((role, rows, cols, num_bits, cols // comps["weight_scale"].shape[-1], remainder,
                     "weight_zero_point" in comps))
    if not geom:
        return None
    num_bits, group_size, has_zero = geom[0][3], geom[0][4], geom[0][6]
    fusable = (num_bits and 32 % num_bits == 0
               and all(r == 0 and nb == num_bits and g == group_size and z == has_zero
                       and c % (32 // num_bits) == 0
                       for _role, _rows, c, nb, g, r, z in geom))
    if not fusable:
        return None
    roles = [g[0] for g in geom]
    flat = {"packed": torch.cat([by_role[r]["weight_packed"].reshape(-1) for r in roles]),
            "scale": torch.cat([by_role[r]["weight_scale"].reshape(-1) for r in roles])}
    if has_zero:
        flat["zero"] = torch.cat([by_role[r]["weight_zero_point"].reshape(-1) for r in roles])
    return {"flat": flat,
            "geom": (num_bits, group_size, tuple((g[0], g[1], g[2]) for g in geom))}


def blob_layout(geom) -> dict:
    """{role: (word offset, scale offset, rows, cols)} inside a blob's flat streams
    (vaayu/packed_expert_kernels.py:301-309)."""
    bits, gs, roles = geom
    out, w_at, s_at = {}, 0, 0
    for role, rows, cols in roles:
        out[role] = (w_at, s_at, rows, cols)
        w_at += rows * cols * bits // 32
        s_at += rows * cols // gs
    return out


def zero_layout(geom) -> dict:
    """{role: word offset of its zero points}: compressed-tensors packs them along rows, so a role
    holds ceil(rows * bits / 32) x (cols / group) words."""
    bits, gs, roles = geom
    per = 32 // bits
    out, at = {}, 0
    for role, rows, cols in roles:
        out[role] = at
        at += -(-rows // per) * (cols // gs)
    return out


def dequantize_expert_blob(blob: dict, dtype: torch.dtype) -> dict:
    """{role: dense weight} from a blob built by `build_expert_blob`: one kernel pass over the
    flat code stream (symmetric blobs) or one per role (zero-point blobs)."""
    num_bits, group_size, roles = blob["geom"]
    flat_packed, flat_scale = blob["flat"]["packed"], blob["flat"]["scale"]
    zero = blob["flat"].get("zero")
    dev = _lib.require_cuda(flat_packed, flat_scale, zero, what="dequantize_expert_blob")
    total = sum(rows * cols for _r, rows, cols in roles)
    flat = torch.empty(total, dtype=dtype, device=dev)
    with torch.cuda.device(dev):
        if zero is None:
            _lib.check(_lib.lib().vy_dequant_flat(
                flat_packed.data_ptr(), flat_packed.numel(), num_bits, flat_scale.data_ptr(),
                _scale_code(flat_scale), group_size, flat.data_ptr(), _act_code(dtype),
                _lib.stream_of(dev)), "dequantize_expert_blob")
        else:
            lay, zl = blob_layout(blob["geom"]), zero_layout(blob["geom"])
            at = 0
            es = flat_scale.element_size()
            for role, rows, cols in roles:
                w_at, s_at, _r, _c = lay[role]
                _lib.check(_lib.lib().vy_dequant_packed_weight(
                    flat_packed.data_ptr() + 4 * w_at, rows, cols, num_bits,
                    flat_scale.data_ptr() + es * s_at, _scale_code(flat_scale), group_size,
                    zero.data_ptr() + 4 * zl[role], flat.data_ptr() + flat.element_size() * at,
                    _act_code(dtype), _lib.stream_of(dev)), "dequantize_expert_blob")
                at += rows * cols
    out, at = {}, 0
    for role, rows, cols in roles:
        out[role] = flat[at:at + rows * cols].view(rows, cols)
        at += rows * cols
    return out


def expert_weights_from_entry(entry: dict, dtype: torch.dtype) -> tuple:
    """(w_gate, w_down, w_up) for one cached expert: a dense entry is already the weights, a
    packed blob is dequantised."""
    dense = entry["dense"] if "dense" in entry else dequantize_expert_blob(entry, dtype)
    return dense["gate"], dense["down"], dense["up"]


def dequantize_expert_weights(by_role: dict, dtype: torch.dtype) -> dict:
    """{role: dense weight} for one expert, in one pass where the blob can be fused."""
    blob = build_expert_blob(by_role)
    if blob is None:
        return {role: dequantize_packed_weight(comps, dtype) for role, comps in by_role.items()}
    return dequantize_expert_blob(blob, dtype)


def accumulate_expert_outputs(final_hidden, contributions) -> None:
    """Add every expert's (expert id, token index, hidden) contribution in EXPERT-ID order, so
    the sum does not depend on the order experts finished in."""
    for _eidx, token_idx, hidden in sorted(contributions, key=lambda c: c[0]):
        final_hidden.index_add_(0, token_idx, hidden.to(final_hidden.dtype))


def route_experts(moe_module, router_logits: torch.Tensor, top_k: int):
    """Combination weights + expert indices for one MoE layer.  The model's own
    `route_tokens_to_experts` when it has one; otherwise softmax -> top-k -> renormalise, on the
    device (vy_moe_topk_softmax).  Returns (weights fp32, indices int64) shaped like the logits
    with E -> top_k."""
    fn = getattr(moe_module, "route_tokens_to_experts", None)
    if callable(fn):
        lead = router_logits.shape[:-1]
        first, second = fn(router_logits.reshape(-1, router_logits.shape[-1]))
        idx, w = (first, second) if not first.is_floating_point() else (second, first)
        return w.reshape(*lead, -1), idx.reshape(*lead, -1)
    return topk_softmax(router_logits, top_k)


def topk_softmax(router_logits: torch.Tensor, top_k: int):
    """softmax(fp32 logits) -> top-k (largest first, ties to the lower id) -> renormalised."""
    dev = _lib.require_cuda(router_logits, what="topk_softmax")
    lead, n_exp = router_logits.shape[:-1], router_logits.shape[-1]
    logits = router_logits.reshape(-1, n_exp)
    if logits.stride(-1) != 1:
        logits = logits.contiguous()
    code = _lib.DTYPE_CODE.get(logits.dtype)
    if code not in (_lib.BF16, _lib.F16, _lib.F32):
        raise NotImplementedError(f"logit dtype {logits.dtype}")
    n = logits.shape[0]
    w = torch.empty(n, top_k, dtype=torch.float32, device=dev)
    idx = torch.empty(n, top_k, dtype=torch.int64, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().vy_moe_topk_softmax(
            logits.data_ptr(), code, logits.stride(0), n, n_exp, top_k, w.data_ptr(),
            idx.data_ptr(), _lib.stream_of(dev)), "topk_softmax")
    return w.reshape(*lead, top_k), idx.reshape(*lead, top_k)


def route_permute(expert_indices: torch.Tensor, num_experts: int) -> dict:
    """The routed gather/permute plan on the device (vy_moe_route_permute): rows (token *
    top_k + slot) grouped by expert id, stable; each token's slots in ascending expert id.
    Returns {"order", "live", "live_start", "slot_order", "n_live", "dropped"} (int32 tensors;
    the counts are 0-d device tensors -- nothing is synchronised)."""
    dev = _lib.require_cuda(expert_indices, what="route_permute")
    ids = expert_indices.contiguous()
    n_tok, top_k = ids.shape if ids.dim() == 2 else (ids.shape[0], 1)
    code = _lib.DTYPE_CODE.get(ids.dtype)
    if code not in (_lib.I32, _lib.I64):
        raise NotImplementedError(f"expert-id dtype {ids.dtype}")
    n = n_tok * top_k
    i32 = dict(dtype=torch.int32, device=dev)
    order, slot = torch.empty(n, **i32), torch.empty(n, **i32)
    live, live_start = torch.empty(num_experts, **i32), torch.empty(num_experts + 1, **i32)
    counters = torch.empty(4, **i32)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().vy_moe_route_permute(
            ids.data_ptr(), code, n_tok, top_k, num_experts, order.data_ptr(), live.data_ptr(),
            live_start.data_ptr(), slot.data_ptr(), counters.data_ptr(), _lib.stream_of(dev)),
            "route_permute")
    return {"order": order, "live": live, "live_start": live_start,
            "slot_order": slot.view(n_tok, top_k), "n_live": counters[0], "dropped": counters[1]}


def compute_expert_dispatch(expert_indices: torch.Tensor, num_experts: int):
    """Permutation-based dispatch: (pair [2, N*top_k] = (token, slot) sorted by expert id,
    stable; starts per expert; counts per expert).  The sort runs on the device; the starts and
    counts come back to the host as lists, like the reference's."""
    plan = route_permute(expert_indices.to(torch.cuda.current_device())
                         if expert_indices.device.type != "cuda" else expert_indices, num_experts)
    top_k = expert_indices.shape[1]
    order = plan["order"].long()
    pair = torch.stack([order // top_k, order % top_k])
    n_live = int(plan["n_live"])
    live = plan["live"][:n_live].long()
    ls = plan["live_start"][:n_live + 1].long()
    counts = torch.zeros(num_experts, dtype=torch.long, device=order.device)
    counts[live] = ls[1:] - ls[:-1]
    starts = counts.cumsum(0) - counts
    return pair, starts.tolist(), counts.tolist()
