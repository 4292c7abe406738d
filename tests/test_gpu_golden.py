"""GPU: the reference's own outputs reproduced by the CUDA path, and the benchmark shapes held to
the oracle.

  - tests/golden/cfg0.npz: configuration 0 (hidden 1024, intermediate 512, 16 experts, top-4,
    4 tokens) through the reference's `stock_experts_prefill(linear=_linear_fp32)` and, for token
    0, `stock_experts_decode` (vaayu/packed_expert_kernels.py:399-410, 780-814);
  - tests/golden/prefill_tiles.npz: `stock_experts_prefill` on 40 tokens of a layer the tiles take
    (hidden 256, intermediate 128, group 32, 8 experts, top-3), fp32 and bf16 routing weights;
  - configuration 2's exact shape (hidden 4096, intermediate 14336, 8 experts, top-2, router
    logits skewed by linspace(0, 0.9, 8)) through the tcgen05 prefill GEMMs, 128 tokens;
  - configuration 1's benchmarked layer (128 experts, top-8, 32 tokens) through the decode GEMVs.
Bars: the reference tests' own (tests/test_packed_prefill_kernels.py:115-175): rel-L2 <= 2e-3
against the fp32-GEMM replay and max |err| <= 2e-2 x RMS; decode rel-L2 <= 1e-3."""
import numpy as np
import pytest
import torch

import vaayu_b200 as vb
from tests import helpers as T
from vaayu_b200 import packed_expert_kernels as pk
from vaayu_b200 import synthetic

pytestmark = pytest.mark.gpu


def _golden_blobs(g, n, hid, inter, bits, gs):
    geom = T.geom(hid, inter, bits, gs)
    return {i: {"geom": geom, "flat": {"packed": torch.from_numpy(g[f"e{i}_packed"].copy()).cuda(),
                                       "scale": T.from_np(g[f"e{i}_scale"], 1).cuda()}}
            for i in range(n)}


@pytest.mark.parametrize("tag", ["fp32", "bf16"])
def test_the_reference_prefill_golden_through_the_kernels(tag):
    g = T.golden("prefill_tiles")
    hid, inter, bits, gs, n_exp, top_k, tokens = (int(v) for v in g["meta"])
    blobs = _golden_blobs(g, n_exp, hid, inter, bits, gs)
    x = T.from_np(g["x"]).cuda()
    w = T.from_np(g[f"w_{tag}"], 0 if tag == "bf16" else None).cuda()
    eidx = torch.from_numpy(g["eidx"].copy())
    ref = g[f"out_{tag}"]
    out = torch.empty(tokens, hid, device="cuda")
    vb.packed_experts_prefill(x, eidx, w, blobs, out, None)                      # the drop-in call
    table = pk.ExpertTable([blobs[i] for i in range(n_exp)])
    for got in (out, vb.moe_forward(x, eidx.cuda(), w, table, path=vb.PATH_PREFILL),
                vb.moe_forward(x, eidx.cuda(), w, table, path=vb.PATH_DECODE)):
        got = got.cpu().numpy()
        assert T.rel_l2(got, ref) <= 2e-3
        assert T.max_abs_over_rms(got, ref) <= 2e-2


def _cfg0():
    g = T.golden("cfg0")
    gen = torch.Generator().manual_seed(0)
    by_roles = [synthetic.make_expert(1024, 512, gen) for _ in range(16)]
    x, w, idx = synthetic.make_tokens(4, 1024, 16, 4, gen)
    assert np.array_equal(T.to_np(idx), g["eidx"]), "synthetic generator drifted from the fixture"
    blobs = [vb.build_expert_blob({r: {k: (v if k == "weight_shape" else v.cuda()) for k, v in c.items()}
                                   for r, c in br.items()}) for br in by_roles]
    return g, blobs, x.cuda(), w.cuda(), idx


def test_configuration_0_reproduces_the_reference_layer():
    g, blobs, x, w, idx = _cfg0()
    table = pk.ExpertTable(blobs)
    out = torch.empty(4, 1024, device="cuda")
    vb.packed_experts_prefill(x, idx, w, dict(enumerate(blobs)), out, None)
    for got in (out, vb.moe_forward(x, idx.cuda(), w, table, path=vb.PATH_DECODE),
                vb.moe_forward(x, idx.cuda(), w, table, path=vb.PATH_PREFILL)):
        got = got.cpu().numpy()
        assert T.rel_l2(got, g["out"]) <= 2e-3
        assert T.max_abs_over_rms(got, g["out"]) <= 2e-2


def test_configuration_0_token_0_reproduces_the_reference_decode():
    g, blobs, x, w, idx = _cfg0()
    order = sorted(range(4), key=lambda s: int(idx[0, s]))
    pairs = [(blobs[int(idx[0, s])], s) for s in order]
    out = torch.empty(1, 1024, device="cuda")
    vb.packed_experts_decode(x[:1], pairs, w[:1], out, None)
    got = out.cpu().numpy()
    assert T.rel_l2(got, g["out_decode_t0"]) <= 1e-3
    assert T.max_abs_over_rms(got, g["out_decode_t0"]) <= 2e-2


def test_configuration_2_shape_through_the_tensor_core_gemms():
    """Hidden 4096, intermediate 14336 (the down GEMM's K: 224 stages), 8 experts, top-2, skewed
    routing, 128 tokens -- the benchmarked prefill layer's shape against the oracle."""
    hid, inter, n_exp, top_k, tokens = 4096, 14336, 8, 2, 128
    gen = torch.Generator().manual_seed(0)
    blobs = []
    for _ in range(n_exp):
        br = synthetic.make_expert(hid, inter, gen)
        blobs.append(vb.build_expert_blob({r: {k: (v if k == "weight_shape" else v.cuda()) for k, v in c.items()}
                                           for r, c in br.items()}))
    x, w, idx = synthetic.make_tokens(tokens, hid, n_exp, top_k, gen, skew=0.9)
    got = vb.moe_forward(x.cuda(), idx.cuda(), w.cuda(), pk.ExpertTable(blobs), path=vb.PATH_PREFILL)
    ref = T.oracle_layer(blobs, x, idx, w)
    got = got.cpu().numpy()
    assert T.rel_l2(got, ref) <= 2e-3
    assert T.max_abs_over_rms(got, ref) <= 2e-2


def test_configuration_1_benchmarked_layer_through_the_gemvs():
    """The bench's layer: 128 experts, top-8, 32 tokens (about 112 experts routed)."""
    hid, inter, n_exp, top_k, tokens = 2048, 768, 128, 8, 32
    gen = torch.Generator().manual_seed(1)
    blobs = []
    for _ in range(n_exp):
        br = synthetic.make_expert(hid, inter, gen)
        blobs.append(vb.build_expert_blob({r: {k: (v if k == "weight_shape" else v.cuda()) for k, v in c.items()}
                                           for r, c in br.items()}))
    x, w, idx = synthetic.make_tokens(tokens, hid, n_exp, top_k, gen)
    got = vb.moe_forward(x.cuda(), idx.cuda(), w.cuda(), pk.ExpertTable(blobs), path=vb.PATH_DECODE)
    ref = T.oracle_layer(blobs, x, idx, w)
    got = got.cpu().numpy()
    assert T.rel_l2(got, ref) <= 1e-3
    assert T.max_abs_over_rms(got, ref) <= 2e-2
