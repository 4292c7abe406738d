"""GPU: the standalone dequant kernels, bit-exact to the reference's own outputs (golden fixtures)
and to the oracle at larger sizes."""
import numpy as np
import pytest
import torch

import vaayu_b200 as vb
from oracle import oracle as O
from tests import helpers as T
from vaayu_b200 import synthetic

pytestmark = pytest.mark.gpu
DT = {0: torch.bfloat16, 1: torch.float16, 2: torch.float32}


def _scale_tensor(arr, code):
    return T.from_np(arr, code).cuda() if code != 2 else torch.from_numpy(arr.copy()).cuda()


def test_unpack_matches_the_reference():
    g = T.golden("unpack")
    for i in range(3):
        rows, cols, bits = (int(v) for v in g[f"c{i}_meta"])
        got = vb.unpack_int32_to_int8(torch.from_numpy(g[f"c{i}_packed"]).cuda(), bits, cols)
        assert np.array_equal(got.cpu().numpy(), g[f"c{i}_codes"]), f"case {i}"


def test_dequantize_packed_weight_is_bit_exact_to_the_reference():
    g = T.golden("dequant_role")
    for i in range(6):
        rows, cols, bits, gs, sc, ac = (int(v) for v in g[f"c{i}_meta"])
        comps = {"weight_packed": torch.from_numpy(g[f"c{i}_packed"]).cuda(),
                 "weight_scale": _scale_tensor(g[f"c{i}_scale"], sc),
                 "weight_shape": torch.tensor([rows, cols])}
        got = vb.dequantize_packed_weight(comps, DT[ac])
        ref = g[f"c{i}_out"]
        assert np.array_equal(T.to_np(got).view(np.uint8), ref.view(np.uint8)), f"case {i}"


def test_blob_dequant_is_bit_exact_to_the_fused_reference_kernel():
    g = T.golden("blob")
    for i in range(3):
        hid, inter, bits, gs, sc, ac = (int(v) for v in g[f"c{i}_meta"])
        blob = {"flat": {"packed": torch.from_numpy(g[f"c{i}_packed"]).cuda(),
                         "scale": _scale_tensor(g[f"c{i}_scale"], sc)},
                "geom": (bits, gs, (("gate", inter, hid), ("down", hid, inter), ("up", inter, hid)))}
        got = vb.dequantize_expert_blob(blob, DT[ac])
        for role in ("gate", "down", "up"):
            assert np.array_equal(T.to_np(got[role]).view(np.uint8), g[f"c{i}_{role}"].view(np.uint8)), \
                f"case {i} {role}"


def test_zero_point_dequant_matches_compressed_tensors():
    g = T.golden("asym")
    for i in range(2):
        rows, cols, bits, gs = (int(v) for v in g[f"c{i}_meta"])
        comps = {"weight_packed": torch.from_numpy(g[f"c{i}_packed"]).cuda(),
                 "weight_scale": T.from_np(g[f"c{i}_scale"]).cuda(),
                 "weight_zero_point": torch.from_numpy(g[f"c{i}_zero"]).cuda(),
                 "weight_shape": torch.tensor([rows, cols])}
        got = vb.dequantize_packed_weight(comps, torch.bfloat16)
        assert np.array_equal(T.to_np(got), g[f"c{i}_out"]), f"case {i}"


@pytest.mark.parametrize("zeros", [False, True])
@pytest.mark.parametrize("sdt,adt", [(torch.float16, torch.bfloat16), (torch.bfloat16, torch.float16),
                                     (torch.float32, torch.bfloat16)])
def test_blob_dequant_matches_the_oracle_at_cfg1_size(zeros, sdt, adt):
    blob = T.make_blobs(2048, 768, 1, gs=128, seed=11, zeros=zeros, scale_dtype=sdt)[0]
    got = vb.dequantize_expert_blob(blob, adt)
    ex = T.oracle_expert(blob)
    lay = O.layout(blob["geom"])
    zl = O.zero_layout(blob["geom"])
    for role, rows, cols in blob["geom"][2]:
        w_at, s_at, _r, _c = lay[role]
        ref = O.dequant_role(ex["packed"][w_at:], rows, cols, 4, ex["scale"][s_at:], T.CODE[sdt], 128,
                             T.CODE[adt], zero=None if ex["zero"] is None else ex["zero"][zl[role]:])
        assert np.array_equal(T.to_np(got[role]).view(np.uint8), ref.view(np.uint8)), role


def test_fp8_block_scaled_is_bit_exact_to_the_reference():
    g = T.golden("fp8")
    for i in range(3):
        rows, cols, sc = (int(v) for v in g[f"c{i}_meta"])
        w = torch.from_numpy(g[f"c{i}_w"]).cuda().view(torch.float8_e4m3fn)
        s = (torch.from_numpy(g[f"c{i}_scale"]).cuda() if sc == 2
             else torch.from_numpy(g[f"c{i}_scale"]).cuda().view(torch.float8_e8m0fnu))
        got = vb.dequantize_block_scaled(w, s)
        assert np.array_equal(T.to_np(got), g[f"c{i}_out"]), f"case {i}"


def test_fp8_block_scaled_cfg4_shape_matches_the_oracle():
    gen = torch.Generator().manual_seed(4)
    w = torch.randn(4096, 14336, generator=gen).to(torch.float8_e4m3fn)
    s = torch.rand(32, 112, generator=gen) * 0.02 + 1e-3
    got = vb.dequantize_block_scaled(w.cuda(), s.cuda())
    ref = O.fp8_dequant(T.to_np(w), s.numpy(), 2)
    assert np.array_equal(T.to_np(got), ref)


def test_fp4_dequant_matches_the_oracle():
    gen = torch.Generator().manual_seed(5)
    w = torch.randint(0, 256, (512, 1024), dtype=torch.uint8, generator=gen)
    s = torch.randint(0, 0x7E, (512, 2048 // 16), dtype=torch.uint8, generator=gen)
    got = vb.dequantize_fp4_block_scaled(w.cuda(), s.cuda())
    ref = O.fp4_dequant(w.numpy(), s.numpy(), 16)
    assert np.array_equal(T.to_np(got), ref)


def test_fp4_dequant_reads_a_float4_x2_container():
    gen = torch.Generator().manual_seed(6)
    w = torch.randint(0, 256, (64, 128), dtype=torch.uint8, generator=gen)
    s = torch.randint(0x30, 0x48, (64, 16), dtype=torch.uint8, generator=gen)
    a = vb.dequantize_fp4_block_scaled(w.cuda().view(torch.float4_e2m1fn_x2),
                                       s.cuda().view(torch.float8_e4m3fn))
    b = vb.dequantize_fp4_block_scaled(w.cuda(), s.cuda())
    assert torch.equal(a, b)


def test_unsupported_dequant_requests_raise():
    comps = synthetic.make_role(64, 128, torch.Generator().manual_seed(1), group=32)
    comps = {k: (v if k == "weight_shape" else v.cuda()) for k, v in comps.items()}
    with pytest.raises(NotImplementedError):
        vb.dequantize_packed_weight(comps, torch.int8)
    comps["weight_g_idx"] = torch.zeros(128, dtype=torch.int32, device="cuda")
    with pytest.raises(NotImplementedError, match="g_idx"):
        vb.dequantize_packed_weight(comps, torch.bfloat16)
