"""The CPU oracle, pinned to archish9/Vaayu's own outputs (tests/golden/, made by
tests/golden/make_golden.py from the reference implementation).

Bit-exact where the reference is exact (unpack, dequant, FP8 block-scaled dequant); within the
reference tests' own bars where the reference sums dot products in an unspecified order
(tests/test_packed_expert_kernels.py:118-168, tests/test_packed_prefill_kernels.py:115-175).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import helpers as T
from vaayu_b200 import synthetic


# ── scalar formats ────────────────────────────────────────────────────────────────────────

def test_fp16_rounding_matches_numpy():
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 10.0 ** rng.integers(-9, 6, 20000),
                           np.array([65504, 65519.99, 65520, 1e-8, 2 ** -24, 2 ** -25, 3 * 2 ** -26,
                                     -0.0, np.inf, -np.inf], np.float32)]).astype(np.float32)
    lib = O.lib()
    got = np.array([lib.vyo_f32_to_f16(float(v)) for v in vals], np.uint16)
    assert np.array_equal(got, vals.astype(np.float16).view(np.uint16))


def test_bf16_rounding_matches_torch():
    rng = np.random.default_rng(1)
    vals = (rng.standard_normal(20000) * 10.0 ** rng.integers(-30, 30, 20000)).astype(np.float32)
    ref = torch.from_numpy(vals).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(O.f32_to_bf16(vals), ref)
    lib = O.lib()
    assert all(lib.vyo_f32_to_bf16(float(v)) == r for v, r in zip(vals[:2000], ref[:2000]))


def test_e4m3_decode_matches_torch_for_every_byte():
    b = np.arange(256, dtype=np.uint8)
    ref = torch.from_numpy(b).view(torch.float8_e4m3fn).float().numpy()
    got = O.e4m3_to_f32(b)
    lib = O.lib()
    got_c = np.array([lib.vyo_e4m3_to_f32(int(v)) for v in b], np.float32)
    both_nan = np.isnan(ref) & np.isnan(got) & np.isnan(got_c)
    assert np.array_equal(got[~both_nan], ref[~both_nan])
    assert np.array_equal(got_c[~both_nan], ref[~both_nan])
    assert both_nan.sum() == np.isnan(ref).sum() == 2


def test_e2m1_table_is_the_ocp_value_set():
    """OCP MX e2m1: sign bit 3, exponent bits 1-2 (bias 1), mantissa bit 0."""
    for nib in range(16):
        s, e, m = nib >> 3, (nib >> 1) & 3, nib & 1
        v = (m / 2.0) if e == 0 else (1 + m / 2.0) * 2.0 ** (e - 1)
        assert O.E2M1[nib] == (-v if s else v)


# ── int-b dequant ─────────────────────────────────────────────────────────────────────────

def test_unpack_convention_matches_the_reference():
    g = T.golden("unpack")
    for i in range(3):
        rows, cols, bits = g[f"c{i}_meta"]
        per = 32 // bits
        words = g[f"c{i}_packed"].astype(np.int64) & 0xFFFFFFFF
        shifts = np.arange(per) * bits
        codes = ((words[..., None] >> shifts) & ((1 << bits) - 1)).reshape(rows, -1)[:, :cols]
        assert np.array_equal(codes - (1 << (bits - 1)), g[f"c{i}_codes"].astype(np.int64))


def test_dequant_role_is_bit_exact_to_dequantize_packed_weight():
    g = T.golden("dequant_role")
    for i in range(6):
        rows, cols, bits, gs, sc, ac = (int(v) for v in g[f"c{i}_meta"])
        scale = g[f"c{i}_scale"]
        if sc == 1:
            scale = scale.view(np.float16)
        got = O.dequant_role(g[f"c{i}_packed"], rows, cols, bits, scale, sc, gs, ac)
        ref = g[f"c{i}_out"]
        if ac == 1:
            ref = ref.view(np.float16)
        assert np.array_equal(got.view(ref.dtype), ref), f"case {i}"


def test_blob_dequant_is_bit_exact_to_the_fused_kernel():
    g = T.golden("blob")
    for i in range(3):
        hid, inter, bits, gs, sc, ac = (int(v) for v in g[f"c{i}_meta"])
        scale = g[f"c{i}_scale"]
        if sc == 1:
            scale = scale.view(np.float16)
        got = O.dequant_flat(g[f"c{i}_packed"], bits, scale, sc, gs, ac)
        ref = np.concatenate([g[f"c{i}_{r}"].reshape(-1) for r in ("gate", "down", "up")])
        if ac == 1:
            ref = ref.view(np.float16)
        assert np.array_equal(got.view(ref.dtype), ref), f"case {i}"
        # the pure-numpy twin agrees with the C code
        twin = O.np_dequant_flat(g[f"c{i}_packed"], bits, T.f32(scale, sc).astype(np.float32),
                                 gs, ac)
        assert np.array_equal(twin, T.f32(got, ac).astype(np.float32))


def test_asymmetric_dequant_matches_compressed_tensors():
    """Where a pin exists (bf16 scales), the zero-point extension is bit-exact to
    compressed-tensors' own `dequantize(x_q, scale, zero_point)`."""
    g = T.golden("asym")
    for i in range(2):
        rows, cols, bits, gs = (int(v) for v in g[f"c{i}_meta"])
        got = O.dequant_role(g[f"c{i}_packed"], rows, cols, bits, g[f"c{i}_scale"], 0, gs, 0,
                             zero=g[f"c{i}_zero"])
        assert np.array_equal(got, g[f"c{i}_out"]), f"case {i}"


def test_zero_point_eight_is_the_symmetric_format():
    gen = torch.Generator().manual_seed(5)
    comps = synthetic.make_role(64, 256, gen, group=32)
    z = torch.full((64, 8), 8, dtype=torch.int32)
    zp = synthetic.pack_zero_points(z)
    args = (T.to_np(comps["weight_packed"]), 64, 256, 4, T.to_np(comps["weight_scale"]), 1, 32, 0)
    assert np.array_equal(O.dequant_role(*args), O.dequant_role(*args, zero=T.to_np(zp)))


# ── FP8 / FP4 ─────────────────────────────────────────────────────────────────────────────

def test_fp8_block_scaled_is_bit_exact_to_the_reference():
    g = T.golden("fp8")
    for i in range(3):
        rows, cols, sc = (int(v) for v in g[f"c{i}_meta"])
        got = O.fp8_dequant(g[f"c{i}_w"], g[f"c{i}_scale"], sc)
        assert np.array_equal(got, g[f"c{i}_out"]), f"case {i}"


def test_fp4_dequant_small_case_by_hand():
    w = np.array([[0x21, 0xF9]], np.uint8)         # nibbles (1,2) and (9,15) -> .5,1, -.5,-6
    scale = np.array([[0x38]], np.uint8)           # e4m3 0x38 = 1.0
    got = T.f32(O.fp4_dequant(w, scale, gs=4))
    assert got.tolist() == [[0.5, 1.0, -0.5, -6.0]]
    scale2 = np.array([[0x40]], np.uint8)          # 2.0
    assert T.f32(O.fp4_dequant(w, scale2, gs=4)).tolist() == [[1.0, 2.0, -1.0, -12.0]]


def test_fp_gemv_is_the_dequantised_product():
    rng = np.random.default_rng(3)
    w = rng.integers(0, 256, (32, 64), dtype=np.uint8)
    w[(w & 0x7F) == 0x7F] = 0                        # no NaN codes
    scale = (rng.random((1, 1)) + 0.5).astype(np.float32)
    x = T.bf16_round_np(rng.standard_normal((2, 64)).astype(np.float32))
    got = T.f32(O.fp_gemv("fp8", w, scale, 2, x))
    deq = T.f32(O.fp8_dequant(w, scale, 2))
    ref = T.f32(T.bf16_round_np((T.f32(x) @ deq.T).astype(np.float32)))
    assert np.array_equal(got, ref)


# ── the layer ─────────────────────────────────────────────────────────────────────────────

def _experts_from(g, n):
    return [{"packed": g[f"e{i}_packed"], "scale": g[f"e{i}_scale"].view(np.float16), "zero": None}
            for i in range(n)]


@pytest.mark.parametrize("tag,wcode", [("fp32", 2), ("bf16", 0)])
def test_decode_layer_matches_stock_experts_decode(tag, wcode):
    g = T.golden("decode")
    hid, inter, bits, gs, k = (int(v) for v in g["meta"])
    experts = _experts_from(g, k)
    slots = g["slots"]
    # pairs sorted by (expert id, slot): expert i is pair i; its weight sits at slot[i]
    out, h = O.moe_layer(T.geom(hid, inter, bits, gs), experts, g["x"], 0,
                         np.arange(k)[None, :], g[f"w_{tag}"], wcode, 1, w_index=slots,
                         want_h=True)
    ref = g[f"out_{tag}"]
    assert T.rel_l2(out, ref) <= 1e-3
    assert T.max_abs_over_rms(out, ref) <= 2e-2
    assert (h == g["h"]).mean() >= 0.99          # stage bar of the reference's own test


def test_decode_down_stage_matches_the_stock_loop():
    g = T.golden("decode")
    hid, inter, bits, gs, k = (int(v) for v in g["meta"])
    experts = _experts_from(g, k)
    # weight 1, fed with stock's own h: y is the rounded down projection
    eq = []
    for i in range(k):
        _out, y = O.moe_layer(T.geom(hid, inter, bits, gs), [experts[i]], g["x"], 0,
                              np.zeros((1, 1), np.int64), np.ones(1, np.float32), 2, 1,
                              want_y=True)
        eq.append(np.mean(T.bf16_round_np(y[0]) == T.bf16_round_np(g["down"][i])))
    assert min(eq) >= 0.98


@pytest.mark.parametrize("tag,wcode", [("fp32", 2), ("bf16", 0)])
def test_prefill_layer_matches_stock_experts_prefill(tag, wcode):
    g = T.golden("prefill")
    hid, inter, bits, gs, n_exp, top_k, tokens = (int(v) for v in g["meta"])
    out = O.moe_layer(T.geom(hid, inter, bits, gs), _experts_from(g, n_exp), g["x"], 0,
                      g["eidx"], g[f"w_{tag}"], wcode, 1)
    ref = g[f"out_{tag}"]
    assert T.rel_l2(out, ref) <= 2e-3            # vs the fp32-GEMM replay
    assert T.rel_l2(out, g["out_flinear"]) <= 1e-2 or tag == "bf16"
    assert T.max_abs_over_rms(out, ref) <= 2e-2


def test_cfg0_layer_matches_the_reference_path():
    """Configuration 0 (symmetric format), inputs regenerated from seed 0."""
    g = T.golden("cfg0")
    gen = torch.Generator().manual_seed(0)
    by_roles = [synthetic.make_expert(1024, 512, gen) for _ in range(16)]
    x, w, idx = synthetic.make_tokens(4, 1024, 16, 4, gen)
    assert np.array_equal(T.to_np(idx), g["eidx"]), "synthetic generator drifted from the fixture"
    experts = [T.expert_from_components(br) for br in by_roles]
    out = O.moe_layer(T.geom(1024, 512), experts, T.to_np(x), 0, T.to_np(idx), T.to_np(w), 2, 1,
                      threads=4)
    assert T.rel_l2(out, g["out"]) <= 2e-3
    assert T.max_abs_over_rms(out, g["out"]) <= 2e-2


@pytest.mark.parametrize("tag,wcode", [("fp32", 2), ("bf16", 0)])
def test_prefill_tiles_layer_matches_stock_experts_prefill(tag, wcode):
    """The 40-token prefill fixture at a geometry the CUDA tiles take (hidden 256, inter 128)."""
    g = T.golden("prefill_tiles")
    hid, inter, bits, gs, n_exp, top_k, tokens = (int(v) for v in g["meta"])
    out = O.moe_layer(T.geom(hid, inter, bits, gs), _experts_from(g, n_exp), g["x"], 0,
                      g["eidx"], g[f"w_{tag}"], wcode, 1)
    ref = g[f"out_{tag}"]
    assert T.rel_l2(out, ref) <= 2e-3
    assert T.max_abs_over_rms(out, ref) <= 2e-2
