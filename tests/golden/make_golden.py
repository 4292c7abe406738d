"""Generate the golden fixtures in tests/golden/ from archish9/Vaayu's OWN implementation.

Run in a container that holds the reference project (read-only) and compressed-tensors:

    python tests/golden/make_golden.py <path to the reference project>

The reference's package `vaayu/__init__.py` pulls in `accelerate`; a namespace stub for `vaayu`
skips that file so `vaayu.moe_patch`, `vaayu.packed_expert_kernels` and the DeepSeek-V4 modeling
module import alone (they only need torch).  Every fixture stores its inputs and the reference's
outputs, except `cfg0_*`, whose inputs are regenerated from the seed by
`vaayu_b200.synthetic` (the npz keeps a checksum of them to catch generator drift).

The GPU test suite and the oracle tests only READ these files; nothing at test time touches the
reference project.
"""
from __future__ import annotations

import hashlib
import sys
import types
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from vaayu_b200 import synthetic  # noqa: E402


def _import_reference(root: Path):
    pkg = types.ModuleType("vaayu")
    pkg.__path__ = [str(root / "vaayu")]
    sys.modules["vaayu"] = pkg
    import vaayu.moe_patch as mp
    import vaayu.packed_expert_kernels as pk
    import vaayu.model_code.deepseek_v4.modeling_deepseek_v4 as ds
    return mp, pk, ds


def bits16(t: torch.Tensor) -> np.ndarray:
    """bf16 / fp16 tensor -> its raw 16-bit patterns."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def arr(t: torch.Tensor) -> np.ndarray:
    if t.dtype in (torch.bfloat16, torch.float16):
        return bits16(t)
    if t.dtype in (torch.float8_e4m3fn, torch.float8_e8m0fnu):
        return t.view(torch.uint8).numpy()
    return t.contiguous().numpy()


DT = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


def checksum(*tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes() if t.dtype != torch.int32
                 else t.contiguous().numpy().tobytes())
    return h.hexdigest()


def quant_pack(ct, weight, bits, gs, scale_dtype):
    """tests/test_packed_expert_dequant.py:44-57's `_reference_pack`, scale dtype selectable."""
    rows, cols = weight.shape
    grouped = weight.reshape(rows, cols // gs, gs).float()
    qmax = 2 ** (bits - 1) - 1
    scale = grouped.abs().amax(dim=-1).clamp(min=1e-6) / qmax
    q = torch.round(grouped / scale.unsqueeze(-1)).clamp(-qmax - 1, qmax).reshape(rows, cols)
    q = q.to(torch.int8)
    return ct.pack_to_int32(q, bits), scale.to(scale_dtype), q


def gen_unpack(mp, ct, out):
    cases = {}
    for i, (rows, cols, bits) in enumerate([(64, 256, 4), (48, 128, 8), (16, 512, 2)]):
        torch.manual_seed(100 + i)
        q = torch.randint(-(1 << (bits - 1)), 1 << (bits - 1), (rows, cols), dtype=torch.int8)
        packed = ct.pack_to_int32(q, bits)
        ref = mp.unpack_int32_to_int8(packed, bits, cols)
        ct_ref = ct.unpack_from_int32(packed, bits, torch.Size([rows, cols]))
        assert torch.equal(ref, ct_ref) and torch.equal(ref, q)
        cases[f"c{i}_packed"] = arr(packed)
        cases[f"c{i}_codes"] = arr(ref)
        cases[f"c{i}_meta"] = np.array([rows, cols, bits])
    np.savez_compressed(out / "unpack.npz", **cases)


def gen_dequant_role(mp, ct, out):
    cases, i = {}, 0
    for rows, cols, bits, gs, sdt, adt in [
            (64, 256, 4, 32, torch.bfloat16, torch.bfloat16),
            (64, 256, 4, 128, torch.float16, torch.bfloat16),
            (32, 512, 4, 128, torch.float16, torch.float16),
            (32, 256, 4, 64, torch.float32, torch.bfloat16),
            (32, 256, 4, 32, torch.float16, torch.float32),
            (32, 256, 8, 64, torch.bfloat16, torch.bfloat16)]:
        torch.manual_seed(200 + i)
        weight = torch.randn(rows, cols, dtype=torch.bfloat16)
        packed, scale, _q = quant_pack(ct, weight, bits, gs, sdt)
        # widen the scale's low bits so the fp16->bf16 rounding of the scale is exercised
        if sdt == torch.float16:
            scale = (torch.rand(scale.shape) * 0.015 + 0.005).to(torch.float16)
        ref = mp.dequantize_packed_weight(
            {"weight_packed": packed, "weight_scale": scale,
             "weight_shape": torch.tensor([rows, cols])}, adt)
        cases[f"c{i}_packed"] = arr(packed)
        cases[f"c{i}_scale"] = arr(scale)
        cases[f"c{i}_out"] = arr(ref)
        cases[f"c{i}_meta"] = np.array([rows, cols, bits, gs, DT[sdt], DT[adt]])
        i += 1
    np.savez_compressed(out / "dequant_role.npz", **cases)


def gen_blob(mp, out):
    cases = {}
    for i, (hid, inter, gs, sdt, adt) in enumerate([
            (128, 64, 32, torch.bfloat16, torch.bfloat16),
            (256, 128, 128, torch.float16, torch.bfloat16),
            (128, 128, 64, torch.float16, torch.float16)]):
        g = torch.Generator().manual_seed(300 + i)
        by_role = synthetic.make_expert(hid, inter, g, group=gs, scale_dtype=sdt)
        blob = mp.build_expert_blob(by_role)
        deq = mp.dequantize_expert_blob(blob, adt)
        cases[f"c{i}_packed"] = arr(blob["flat"]["packed"])
        cases[f"c{i}_scale"] = arr(blob["flat"]["scale"])
        for role in ("gate", "down", "up"):
            cases[f"c{i}_{role}"] = arr(deq[role])
        cases[f"c{i}_meta"] = np.array([hid, inter, 4, gs, DT[sdt], DT[adt]])
    np.savez_compressed(out / "blob.npz", **cases)


def _experts(mp, hid, inter, n, gs, seed, sdt=torch.float16):
    g = torch.Generator().manual_seed(seed)
    return [mp.build_expert_blob(synthetic.make_expert(hid, inter, g, group=gs, scale_dtype=sdt))
            for _ in range(n)]


def gen_decode(mp, pk, out):
    """stock_experts_decode at one token, fp32 and bf16 routing weights, plus its stages."""
    cases = {}
    hid, inter, gs, k = 256, 128, 32, 6
    blobs = _experts(mp, hid, inter, k, gs, 400)
    g = torch.Generator().manual_seed(401)
    x = (torch.randn(1, hid, generator=g) * 0.5).to(torch.bfloat16)
    w = torch.rand(1, k, generator=g) + 0.05
    w = w / w.sum(-1, keepdim=True)
    slots = torch.randperm(k, generator=g).tolist()
    pairs = [(blobs[i], slots[i]) for i in range(k)]
    for tag, rw in (("fp32", w), ("bf16", w.to(torch.bfloat16))):
        o = torch.empty(1, hid)
        pk.stock_experts_decode(x, pairs, rw, o, F.silu)
        cases[f"out_{tag}"] = arr(o)
        cases[f"w_{tag}"] = arr(rw)
    hs, downs = [], []
    for blob, _s in pairs:
        wg, wd, wu = mp.expert_weights_from_entry(blob, x.dtype)
        h = F.silu(F.linear(x, wg)) * F.linear(x, wu)
        hs.append(arr(h)[0])
        downs.append(arr(F.linear(h, wd).float())[0])
    cases["h"] = np.stack(hs)
    cases["down"] = np.stack(downs)
    cases["x"] = arr(x)
    cases["slots"] = np.array(slots)
    for i, blob in enumerate(blobs):
        cases[f"e{i}_packed"] = arr(blob["flat"]["packed"])
        cases[f"e{i}_scale"] = arr(blob["flat"]["scale"])
    cases["meta"] = np.array([hid, inter, 4, gs, k])
    np.savez_compressed(out / "decode.npz", **cases)


def gen_prefill(mp, pk, out, name="prefill", hid=128, inter=64, gs=32, tokens=12):
    """stock_experts_prefill with fp32-summed GEMMs (the kernels' reference) and with F.linear.
    `prefill` (intermediate 64) pins the oracle; `prefill_tiles` (hidden 256, intermediate 128,
    40 tokens) is a geometry the CUDA kernels take, so the GPU suite reproduces it directly."""
    cases = {}
    n_exp, top_k = 8, 3
    blobs = _experts(mp, hid, inter, n_exp, gs, 500)
    g = torch.Generator().manual_seed(501)
    eidx = torch.stack([torch.randperm(n_exp, generator=g)[:top_k] for _ in range(tokens)])
    x = (torch.randn(tokens, hid, generator=g) * 0.5).to(torch.bfloat16)
    w = torch.rand(tokens, top_k, generator=g) + 0.05
    w = w / w.sum(-1, keepdim=True)
    bmap = dict(enumerate(blobs))
    for tag, rw in (("fp32", w), ("bf16", w.to(torch.bfloat16))):
        o = torch.empty(tokens, hid)
        pk.stock_experts_prefill(x, eidx, rw, bmap, o, F.silu, linear=pk._linear_fp32)
        cases[f"out_{tag}"] = arr(o)
        cases[f"w_{tag}"] = arr(rw)
    o = torch.empty(tokens, hid)
    pk.stock_experts_prefill(x, eidx, w, bmap, o, F.silu)
    cases["out_flinear"] = arr(o)
    cases["x"] = arr(x)
    cases["eidx"] = arr(eidx)
    for i, blob in enumerate(blobs):
        cases[f"e{i}_packed"] = arr(blob["flat"]["packed"])
        cases[f"e{i}_scale"] = arr(blob["flat"]["scale"])
    cases["meta"] = np.array([hid, inter, 4, gs, n_exp, top_k, tokens])
    # the host-side plan of vaayu/packed_expert_kernels.py:676-717 on this routing
    order, live, counts = pk._prefill_plan(eidx)
    cases["plan_order"] = arr(order)
    cases["plan_live"] = arr(live)
    cases["plan_counts"] = arr(counts)
    cases["slot_order"] = arr(torch.argsort(eidx, dim=1, stable=True)
                              + (torch.arange(tokens) * top_k)[:, None])
    np.savez_compressed(out / f"{name}.npz", **cases)


def gen_cfg0(mp, pk, out):
    """Configuration 0 (hidden 1024, inter 512, 16 experts, top-4, 4 tokens), symmetric format,
    through the reference's own CPU path.  Inputs are regenerated from seed 0 by
    vaayu_b200.synthetic; the checksum pins them."""
    hid, inter, n_exp, top_k, tokens = 1024, 512, 16, 4, 4
    g = torch.Generator().manual_seed(0)
    by_roles = [synthetic.make_expert(hid, inter, g) for _ in range(n_exp)]
    x, w, idx = synthetic.make_tokens(tokens, hid, n_exp, top_k, g)
    blobs = {e: mp.build_expert_blob(br) for e, br in enumerate(by_roles)}
    o = torch.empty(tokens, hid)
    pk.stock_experts_prefill(x, idx, w, blobs, o, F.silu, linear=pk._linear_fp32)
    o1 = torch.empty(1, hid)
    pairs = [(blobs[int(idx[0, s])], s) for s in sorted(range(top_k), key=lambda s: int(idx[0, s]))]
    pk.stock_experts_decode(x[:1], pairs, w[:1], o1, F.silu)
    csum = checksum(*[blobs[e]["flat"]["packed"] for e in range(n_exp)],
                    *[blobs[e]["flat"]["scale"] for e in range(n_exp)], x, w, idx)
    np.savez_compressed(out / "cfg0.npz", out=arr(o), out_decode_t0=arr(o1), eidx=arr(idx),
                        w=arr(w), checksum=np.array(csum))


def gen_fp8(ds, out):
    cases = {}
    for i, (shape, block, sdt) in enumerate([((256, 256), (128, 128), torch.float32),
                                             ((64, 128), (32, 64), torch.float8_e8m0fnu),
                                             ((128, 384), (128, 128), torch.float32)]):
        torch.manual_seed(600 + i)
        weight = torch.randn(*shape).to(torch.float8_e4m3fn)
        if sdt == torch.float32:
            scale = torch.rand(shape[0] // block[0], shape[1] // block[1]) * 0.02 + 1e-3
        else:
            scale = torch.randn(shape[0] // block[0], shape[1] // block[1]).exp().to(sdt)
        ref = ds.dequantize_block_scaled(weight, scale)
        cases[f"c{i}_w"] = arr(weight)
        cases[f"c{i}_scale"] = arr(scale)
        cases[f"c{i}_out"] = arr(ref)
        cases[f"c{i}_meta"] = np.array([shape[0], shape[1], 2 if sdt == torch.float32 else 4])
    np.savez_compressed(out / "fp8.npz", **cases)


def gen_asym(ct, out):
    """compressed-tensors' own `dequantize(x_q, scale, zero_point)` on unpacked zero points, with
    bf16 scales: there its order of operations equals the extension's (scale in the activation
    dtype, (q - zp) exact), so this pins the asymmetric format's bits where a pin exists."""
    from compressed_tensors.quantization.lifecycle.forward import dequantize
    cases = {}
    for i, (rows, cols, gs) in enumerate([(64, 256, 32), (40, 256, 128)]):
        g = torch.Generator().manual_seed(700 + i)
        comps = synthetic.make_role(rows, cols, g, group=gs, zeros=True, scale_dtype=torch.bfloat16)
        packed, scale, zp_packed = (comps["weight_packed"], comps["weight_scale"],
                                    comps["weight_zero_point"])
        q = ct.unpack_from_int32(packed, 4, torch.Size([rows, cols]))
        zp = ct.unpack_from_int32(zp_packed, 4, torch.Size([rows, cols // gs]), packed_dim=0)
        ref = dequantize(q, scale, zp, dtype=torch.bfloat16)
        cases[f"c{i}_packed"] = arr(packed)
        cases[f"c{i}_scale"] = arr(scale)
        cases[f"c{i}_zero"] = arr(zp_packed)
        cases[f"c{i}_out"] = arr(ref)
        cases[f"c{i}_meta"] = np.array([rows, cols, 4, gs])
    np.savez_compressed(out / "asym.npz", **cases)


def main():
    if len(sys.argv) < 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <path to the reference project> [fixture ...]")
    root = Path(sys.argv[1])
    mp, pk, ds = _import_reference(root)
    import compressed_tensors.compressors.pack_quantized.helpers as ct
    torch.set_num_threads(8)
    gens = {
        "unpack": lambda: gen_unpack(mp, ct, HERE),
        "dequant_role": lambda: gen_dequant_role(mp, ct, HERE),
        "blob": lambda: gen_blob(mp, HERE),
        "decode": lambda: gen_decode(mp, pk, HERE),
        "prefill": lambda: gen_prefill(mp, pk, HERE),
        "prefill_tiles": lambda: gen_prefill(mp, pk, HERE, "prefill_tiles", 256, 128, 32, 40),
        "cfg0": lambda: gen_cfg0(mp, pk, HERE),
        "fp8": lambda: gen_fp8(ds, HERE),
        "asym": lambda: gen_asym(ct, HERE),
    }
    for name in sys.argv[2:] or list(gens):
        gens[name]()
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
