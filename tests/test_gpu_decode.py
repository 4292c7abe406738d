"""GPU: the decode kernels (token-batched int4 GEMV) against the oracle and the reference's own
goldens, with the reference tests' bars (tests/test_packed_expert_kernels.py:118-298)."""
import numpy as np
import pytest
import torch

import vaayu_b200 as vb
from tests import helpers as T
from vaayu_b200 import packed_expert_kernels as pk

pytestmark = pytest.mark.gpu

# (hidden, intermediate, group, top_k): the reference test's two int4 geometries, and cfg1's
GEOMS = [pytest.param(2048, 512, 32, 10, id="qwen3next-int4-g32"),
         pytest.param(3072, 1536, 128, 8, id="minimax-like-int4-g128"),
         pytest.param(2048, 768, 128, 8, id="cfg1-qwen3-30b-a3b")]


def _case(hid, inter, gs, k, seed=0, w_dtype=torch.float32, zeros=False):
    """(x, pairs, w, blobs): expert i (ascending id) routed in a shuffled slot."""
    blobs = T.make_blobs(hid, inter, k, gs=gs, seed=hid + inter + gs, zeros=zeros)
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(1, hid, generator=g) * 0.5).to(torch.bfloat16).cuda()
    w = torch.rand(1, k, generator=g) + 0.05
    w = (w / w.sum(-1, keepdim=True)).to(w_dtype).cuda()
    slots = torch.randperm(k, generator=g).tolist()
    return x, [(blobs[i], slots[i]) for i in range(k)], w, blobs, slots


def _run(x, pairs, w):
    out = torch.full((1, x.shape[1]), float("nan"), device="cuda")
    vb.packed_experts_decode(x, pairs, w, out, None)
    torch.cuda.synchronize()
    return out


def _oracle(x, blobs, slots, w, **kw):
    k = len(blobs)
    return T.oracle_layer(blobs, x, torch.arange(k).view(1, k), w, w_index=slots, **kw)


def test_decode_matches_the_reference_golden():
    g = T.golden("decode")
    hid, inter, bits, gs, k = (int(v) for v in g["meta"])
    blobs = [{"flat": {"packed": torch.from_numpy(g[f"e{i}_packed"]).cuda(),
                       "scale": torch.from_numpy(g[f"e{i}_scale"].view(np.float16)).cuda()},
              "geom": T.geom(hid, inter, bits, gs)} for i in range(k)]
    x = T.from_np(g["x"]).cuda()
    pairs = [(blobs[i], int(g["slots"][i])) for i in range(k)]
    for tag, dt in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
        w = T.from_np(g[f"w_{tag}"]).cuda() if dt == torch.bfloat16 else torch.from_numpy(g[f"w_{tag}"]).cuda()
        got = _run(x, pairs, w)
        ref = g[f"out_{tag}"]
        assert T.rel_l2(got.cpu().numpy(), ref) <= 1e-3
        assert T.max_abs_over_rms(got.cpu().numpy(), ref) <= 2e-2
    h = torch.empty(k, inter, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(1, hid, device="cuda")
    pk._launch(x, pairs, torch.from_numpy(g["w_fp32"]).cuda(), out, h_out=h)
    torch.cuda.synchronize()
    assert (T.to_np(h) == g["h"]).mean() >= 0.99


@pytest.mark.parametrize("hid,inter,gs,k", GEOMS)
def test_each_rounding_point_matches_the_oracle(hid, inter, gs, k):
    """Stage by stage: h (gate/up/SiLU/product) and the down output (weight 1) rounded where the
    stock loop rounds; only the order inside each dot product may differ."""
    x, pairs, w, blobs, slots = _case(hid, inter, gs, k)
    h = torch.empty(k, inter, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(1, hid, device="cuda")
    pk._launch(x, pairs, w, out, h_out=h)
    ones = torch.ones(1, k, device="cuda")
    contrib = torch.empty(k, hid, device="cuda")
    table = pk.ExpertTable(blobs)
    vb.moe_forward(x, torch.arange(k, device="cuda").view(1, k), ones, table, contrib=contrib)
    torch.cuda.synchronize()
    _o, h_ref = _oracle(x, blobs, list(range(k)), ones, want_h=True)
    assert (T.to_np(h) == h_ref).mean() >= 0.99, "gate/up/SiLU/product stage"
    # the down stage alone: the oracle is fed the kernel's own h
    _o, y_ref = _oracle(x, blobs, list(range(k)), ones, want_y=True, h_in=T.to_np(h))
    assert (contrib.cpu().numpy() == y_ref).mean() >= 0.99, "down stage"


@pytest.mark.parametrize("w_dtype", [torch.float32, torch.bfloat16], ids=["fp32-w", "bf16-w"])
def test_the_expert_sum_runs_in_table_order(w_dtype):
    """EXACT: out = the fp32 sum, in table order, of each pair's own contribution."""
    x, pairs, w, blobs, slots = _case(2048, 512, 32, 10, w_dtype=w_dtype)
    full = _run(x, pairs, w)
    k = len(pairs)
    contrib = torch.empty(k, 2048, device="cuda")
    ids = torch.arange(k, device="cuda", dtype=torch.int32).view(1, k)
    w_idx = torch.tensor(slots, dtype=torch.int32, device="cuda")
    vb.moe_forward(x, ids, w, pk.ExpertTable(blobs), contrib=contrib, w_index=w_idx)
    c = contrib.cpu().numpy()
    expected = np.zeros(2048, np.float32)
    for i in range(k):
        expected = (expected + c[i]).astype(np.float32)
    assert np.array_equal(full.cpu().numpy()[0], expected)


@pytest.mark.parametrize("hid,inter,gs,k", GEOMS)
def test_kernel_output_is_as_accurate_as_the_stock_arithmetic(hid, inter, gs, k):
    x, pairs, w, blobs, slots = _case(hid, inter, gs, k)
    got = _run(x, pairs, w).cpu().numpy()
    ref = _oracle(x, blobs, slots, w)
    assert T.rel_l2(got, ref) <= 1e-3
    assert T.max_abs_over_rms(got, ref) <= 2e-2
    ids = torch.zeros(1, k, dtype=torch.long)
    ids[0, torch.tensor(slots)] = torch.arange(k)
    truth = T.fp64_layer(blobs, x, ids, w)
    assert T.rel_l2(got, truth) <= 1.25 * T.rel_l2(ref, truth) + 1e-12


def test_bf16_routing_weights_round_like_the_stock_loop():
    x, pairs, w, blobs, slots = _case(2048, 512, 32, 10, w_dtype=torch.bfloat16)
    got = _run(x, pairs, w).cpu().numpy()
    ref = _oracle(x, blobs, slots, w)
    assert (T.bf16_round_np(got) == T.bf16_round_np(ref)).mean() >= 0.99
    assert T.rel_l2(got, ref) <= 1e-3


def test_the_output_does_not_depend_on_where_the_blobs_live():
    x, pairs, w, blobs, slots = _case(2048, 512, 32, 10)
    clones = [({"flat": {n: t.clone() for n, t in b["flat"].items()}, "geom": b["geom"]}, s)
              for b, s in pairs]
    assert torch.equal(_run(x, pairs, w), _run(x, clones, w))


def test_a_zero_weight_duplicate_slot_changes_nothing():
    x, pairs, w, blobs, slots = _case(2048, 512, 32, 10)
    k = w.shape[1]
    w2 = torch.cat([w, torch.zeros(1, 1, dtype=w.dtype, device=w.device)], dim=1)
    dup = pairs[:1] + [(pairs[0][0], k)] + pairs[1:]
    assert torch.equal(_run(x, pairs, w), _run(x, dup, w2))


def test_back_to_back_calls_do_not_share_a_table():
    cases = [_case(2048, 512, 32, 10, seed=s) for s in range(12)]
    outs = []
    for x, pairs, w, _b, _s in cases:
        out = torch.empty(1, x.shape[1], device="cuda")
        vb.packed_experts_decode(x, pairs, w, out, None)
        outs.append(out)
    torch.cuda.synchronize()
    for (x, pairs, w, _b, _s), out in zip(cases, outs):
        assert torch.equal(out, _run(x, pairs, w))


def test_a_nan_inside_the_experts_is_not_masked():
    x, pairs, w, blobs, slots = _case(2048, 512, 32, 10)
    x = x.clone()
    x[0, 5] = float("nan")
    assert torch.isnan(_run(x, pairs, w)).all()


def test_an_unsupported_geometry_raises_instead_of_falling_back():
    x, pairs, w, blobs, slots = _case(192, 96, 32, 2)
    with pytest.raises(NotImplementedError):
        _run(x, pairs, w)


def test_a_call_mixing_geometries_raises_instead_of_falling_back():
    x, pairs, w, blobs, slots = _case(2048, 512, 32, 10)
    other = T.make_blobs(2048, 512, 1, gs=64, seed=9)[0]
    with pytest.raises(NotImplementedError, match="one geometry"):
        _run(x, pairs[:9] + [(other, pairs[9][1])], w)
    dense = {"dense": dict(zip(("gate", "down", "up"), vb.expert_weights_from_entry(blobs[0], x.dtype)))}
    with pytest.raises(NotImplementedError):
        _run(x, [(dense, pairs[0][1])] + pairs[1:], w)


# ── token-batched decode through the resident table (device routing, no host sync) ────────

def _batched(hid, inter, gs, n_exp, top_k, tokens, seed=0, zeros=False, act=torch.bfloat16,
             w_dtype=torch.float32):
    blobs = T.make_blobs(hid, inter, n_exp, gs=gs, seed=seed + 100, zeros=zeros)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(tokens, hid, generator=g).to(act).cuda()
    w, idx = torch.topk(torch.randn(tokens, n_exp, generator=g).softmax(-1), top_k, -1)
    w = (w / w.sum(-1, keepdim=True)).to(w_dtype).cuda()
    return blobs, x, idx.cuda(), w


@pytest.mark.parametrize("tokens", [1, 8, 32, 64])
def test_batched_decode_matches_the_oracle(tokens):
    blobs, x, idx, w = _batched(2048, 768, 128, 32, 8, tokens)
    got = vb.moe_forward(x, idx, w, pk.ExpertTable(blobs), path=vb.PATH_DECODE).cpu().numpy()
    ref = T.oracle_layer(blobs, x, idx, w)
    assert T.rel_l2(got, ref) <= 1e-3
    assert T.max_abs_over_rms(got, ref) <= 2e-2
    assert (T.bf16_round_np(got) == T.bf16_round_np(ref)).mean() >= 0.99


def test_many_tokens_on_one_expert_take_several_passes():
    """64 tokens all routed to the same 4 experts: 64 columns per expert, two 32-token passes."""
    blobs, x, idx, w = _batched(1024, 512, 128, 8, 4, 64, seed=3)
    idx = torch.arange(4, device="cuda").repeat(64, 1)
    got = vb.moe_forward(x, idx, w, pk.ExpertTable(blobs), path=vb.PATH_DECODE).cpu().numpy()
    assert T.rel_l2(got, T.oracle_layer(blobs, x, idx, w)) <= 1e-3


def test_zero_point_layer_matches_the_oracle():
    blobs, x, idx, w = _batched(1024, 512, 128, 16, 4, 4, seed=7, zeros=True)
    got = vb.moe_forward(x, idx, w, pk.ExpertTable(blobs), path=vb.PATH_DECODE).cpu().numpy()
    ref = T.oracle_layer(blobs, x, idx, w)
    assert T.rel_l2(got, ref) <= 1e-3 and T.max_abs_over_rms(got, ref) <= 2e-2


def test_fp16_activations_match_the_oracle():
    blobs, x, idx, w = _batched(1024, 512, 64, 16, 4, 8, seed=8, act=torch.float16,
                                w_dtype=torch.float16)
    got = vb.moe_forward(x, idx, w, pk.ExpertTable(blobs), path=vb.PATH_DECODE).cpu().numpy()
    ref = T.oracle_layer(blobs, x, idx, w)
    assert T.rel_l2(got, ref) <= 1e-3


def test_a_token_does_not_depend_on_its_batch():
    blobs, x, idx, w = _batched(2048, 768, 128, 32, 8, 24, seed=2)
    table = pk.ExpertTable(blobs)
    full = vb.moe_forward(x, idx, w, table, path=vb.PATH_DECODE)
    for t in (0, 11, 23):
        alone = vb.moe_forward(x[t:t + 1], idx[t:t + 1], w[t:t + 1], table, path=vb.PATH_DECODE)
        assert torch.equal(alone[0], full[t])


def test_strided_inputs_and_outputs_are_read_as_what_they_hold():
    blobs, x, idx, w = _batched(1024, 512, 128, 16, 4, 8, seed=4)
    table = pk.ExpertTable(blobs)
    dense = vb.moe_forward(x, idx, w, table, path=vb.PATH_DECODE)
    wide_x = torch.zeros(8, 2048, dtype=x.dtype, device="cuda")
    wide_x[:, 512:1536] = x
    wide_w = torch.zeros(8, 12, device="cuda")
    wide_w[:, 3:7] = w
    wide_o = torch.full((8, 3000), 7.0, device="cuda")
    out = wide_o[:, 1000:2024]
    vb.moe_forward(wide_x[:, 512:1536], idx, wide_w[:, 3:7], table, out=out, path=vb.PATH_DECODE)
    assert torch.equal(out, dense)
    assert (wide_o[:, :1000] == 7.0).all() and (wide_o[:, 2024:] == 7.0).all()


def test_an_expert_id_outside_the_table_is_dropped():
    blobs, x, idx, w = _batched(1024, 512, 128, 8, 2, 4, seed=5)
    table = pk.ExpertTable(blobs)
    bad = idx.clone()
    bad[1, 1] = 99
    got = vb.moe_forward(x, bad, w, table, path=vb.PATH_DECODE)
    w2 = w.clone()
    w2[1, 1] = 0.0
    ref = vb.moe_forward(x, idx, w2, table, path=vb.PATH_DECODE)
    assert torch.equal(got[0], ref[0]) and torch.equal(got[2:], ref[2:])
    assert torch.allclose(got[1], ref[1], rtol=0, atol=1e-6)


def test_global_ids_with_an_expert_base_read_through_a_strided_view():
    """A rank's table holds experts [16, 32) of a global id space: ids outside it drop their
    slot; the ids may sit in a wider buffer (row stride > top_k)."""
    blobs, x, idx, w = _batched(1024, 512, 128, 32, 4, 24, seed=11)
    local = pk.ExpertTable(blobs[16:32])
    wide = torch.full((24, 9), -7, dtype=torch.int32, device="cuda")
    wide[:, 2:6] = idx.to(torch.int32)
    got = vb.moe_forward(x, wide[:, 2:6], w, local, path=vb.PATH_DECODE, expert_base=16)
    masked = torch.where((idx >= 16) & (idx < 32), idx - 16, torch.full_like(idx, -1))
    ref = vb.moe_forward(x, masked, w, local, path=vb.PATH_DECODE)
    assert torch.equal(got, ref)


@pytest.mark.parametrize("col_blocks", [1, 2, 4])
def test_the_column_block_count_does_not_change_a_bit(col_blocks):
    """More passes per expert (col_blocks=1: 8 tokens per pass) or fewer: same per-row math."""
    blobs, x, idx, w = _batched(2048, 768, 128, 8, 4, 40, seed=12)
    table = pk.ExpertTable(blobs)
    ref = vb.moe_forward(x, idx, w, table, path=vb.PATH_DECODE)
    got = vb.moe_forward(x, idx, w, table, path=vb.PATH_DECODE, col_blocks=col_blocks)
    assert torch.equal(got, ref)


def test_ordered_partial_sum():
    from vaayu_b200 import _lib
    g = torch.Generator().manual_seed(3)
    parts = (torch.randn(5, 32, 2048, generator=g) * torch.logspace(-3, 3, 5).reshape(5, 1, 1)).cuda()
    out = torch.empty(32, 2048, device="cuda")
    _lib.check(_lib.lib().vy_sum_ordered(parts.data_ptr(), 5, out.numel(), out.data_ptr(),
                                         _lib.stream_of(out.device)), "vy_sum_ordered")
    ref = parts[0].clone()
    for q in range(1, 5):
        ref += parts[q]
    assert torch.equal(out, ref)


@pytest.mark.parametrize("hid,inter,tokens", [pytest.param(7168, 2048, 8, id="deepseek-v3-dims"),
                                              pytest.param(3072, 1536, 80, id="four-column-blocks")])
def test_down_grids_larger_than_one_resident_wave(hid, inter, tokens):
    """DeepSeek-V3-shaped rows (448 down tiles) and a 4-column-block call (one CTA per SM): the
    down kernel loops its resident grid over more (tile, chunk) items than it has CTAs."""
    blobs, x, idx, w = _batched(hid, inter, 128, 16, 4, tokens, seed=13)
    got = vb.moe_forward(x, idx, w, pk.ExpertTable(blobs), path=vb.PATH_DECODE).cpu().numpy()
    ref = T.oracle_layer(blobs, x, idx, w)
    assert T.rel_l2(got, ref) <= 1e-3
    assert T.max_abs_over_rms(got, ref) <= 2e-2


def test_a_layer_read_from_a_checkpoint_computes_the_same_output(tmp_path):
    from vaayu_b200 import checkpoint as ck
    from vaayu_b200 import synthetic
    g = torch.Generator().manual_seed(31)
    tensors, blobs = {}, []
    for e in range(8):
        by_role = synthetic.make_expert(1024, 512, g, group=128)
        for role, seg in (("gate", "gate_proj"), ("down", "down_proj"), ("up", "up_proj")):
            for comp, t in by_role[role].items():
                tensors[f"model.layers.0.mlp.experts.{e}.{seg}.{comp}"] = t
        blobs.append(vb.build_expert_blob({r: {k: (v if k == "weight_shape" else v.cuda()) for k, v in c.items()}
                                           for r, c in by_role.items()}))
    ck.write_safetensors(str(tmp_path / "m.safetensors"), tensors)
    cp = ck.Checkpoint(str(tmp_path / "m.safetensors"))
    try:
        table = cp.layer_table("model.layers.0.mlp")
        x = torch.randn(6, 1024, generator=g).to(torch.bfloat16).cuda()
        w, idx = torch.topk(torch.randn(6, 8, generator=g).softmax(-1), 2, -1)
        w, idx = w.cuda(), idx.cuda()
        assert torch.equal(vb.moe_forward(x, idx, w, table, path=vb.PATH_DECODE),
                           vb.moe_forward(x, idx, w, pk.ExpertTable(blobs), path=vb.PATH_DECODE))
    finally:
        cp.close()


@pytest.mark.parametrize("gated", [False, True], ids=["deepseek-ungated", "qwen-sigmoid-gated"])
def test_the_shared_expert_joins_like_the_model_epilogue(gated):
    """result = routed_sum.to(bf16) + shared.to(bf16); gated: sigmoid(gate) * shared in bf16."""
    routed, x, idx, w = _batched(1024, 512, 128, 8, 2, 10, seed=17)
    shared = T.make_blobs(1024, 512, 1, gs=128, seed=99)
    gate = torch.sigmoid(torch.randn(10, 1, generator=torch.Generator().manual_seed(5))).to(torch.bfloat16).cuda() \
        if gated else None
    got = vb.moe_forward_with_shared(x, idx, w, pk.ExpertTable(routed), pk.ExpertTable(shared), gate=gate)
    r = torch.from_numpy(T.oracle_layer(routed, x, idx, w))
    sh_w = gate.float().cpu() if gated else torch.ones(10, 1)
    s = torch.from_numpy(T.oracle_layer(shared, x, torch.zeros(10, 1, dtype=torch.long),
                                        sh_w.to(torch.bfloat16) if gated else sh_w))
    ref = (r.to(torch.bfloat16) + s.to(torch.bfloat16)).float().numpy()
    g = got.float().cpu().numpy()
    assert got.dtype == torch.bfloat16
    assert T.rel_l2(g, ref) <= 2e-3
    # each bf16 term (routed sum, shared output) may sit one bf16 step from the oracle's, and the
    # sum rounds once more: at most 2^-7 of |routed| + |shared| + |result| (cancellation included)
    rb, sb = r.to(torch.bfloat16).float().numpy(), s.to(torch.bfloat16).float().numpy()
    rms = float(np.sqrt(np.mean(ref ** 2)))
    bound = 2.0 ** -7 * (np.abs(rb) + np.abs(sb) + np.abs(ref)) + 1e-3 * rms
    assert np.all(np.abs(g - ref) <= bound)


@pytest.mark.parametrize("path", [vb.PATH_DECODE, vb.PATH_PREFILL], ids=["decode", "prefill"])
@pytest.mark.parametrize("gated", [False, True], ids=["ungated", "gated"])
@pytest.mark.parametrize("wdt", [torch.float32, torch.bfloat16], ids=["w-fp32", "w-bf16"])
def test_the_fused_shared_expert_equals_two_calls_bit_for_bit(path, gated, wdt):
    """One layer call with the shared expert as every token's extra slot (shared_last) equals the
    routed layer and the shared expert as separate calls on the same path, joined by the model's
    epilogue out.to(bf16) + shared.to(bf16) -- bit for bit, the routed fp32 sum included."""
    if path == vb.PATH_PREFILL and not pk.prefill_available():
        pytest.skip("prefill kernels not built")
    routed, x, idx, w = _batched(1024, 512, 128, 8, 2, 37, seed=23)
    w = w.to(wdt)
    shared = pk.ExpertTable(T.make_blobs(1024, 512, 1, gs=128, seed=77))
    table = pk.ExpertTable(routed)
    gate = torch.sigmoid(torch.randn(37, 1, generator=torch.Generator().manual_seed(9))).to(torch.bfloat16).cuda() \
        if gated else None
    out = torch.empty(37, 1024, device="cuda")
    got = vb.moe_forward_with_shared(x, idx, w, table, shared, gate=gate, out=out, path=path)
    r = vb.moe_forward(x, idx, w, table, path=path)
    sw = gate.reshape(37, 1) if gated else torch.ones(37, 1, device="cuda")
    s = vb.moe_forward(x, torch.zeros(37, 1, dtype=torch.int32, device="cuda"), sw, shared, path=path)
    assert got.dtype == torch.bfloat16
    assert torch.equal(out, r)
    assert torch.equal(got, r.to(torch.bfloat16) + s.to(torch.bfloat16))
    # the two-call form of the same API agrees too
    two = vb.moe_forward_with_shared(x, idx, w, table, shared, gate=gate, path=path, fused=False)
    if path == vb.PATH_DECODE:
        assert torch.equal(got, two)


@pytest.mark.parametrize("tokens", [1, 3])
def test_split_k_gate_up_is_bit_identical_to_one_warp_per_unit(tokens):
    """Few-token calls share each gate/up unit's K range among warps; the per-stage partial dots
    are added in stage order by the last split, so every split count gives the same bits."""
    blobs, x, idx, w = _batched(2048, 768, 128, 64, 8, tokens, seed=31)
    table = pk.ExpertTable(blobs)
    outs = {s: vb.moe_forward(x, idx, w, table, path=vb.PATH_DECODE, k_splits=s) for s in (1, 2, 4, 8)}
    auto = vb.moe_forward(x, idx, w, table, path=vb.PATH_DECODE)
    for s in (2, 4, 8):
        assert torch.equal(outs[s], outs[1]), f"k_splits={s}"
    assert torch.equal(auto, outs[1])
    ref = T.oracle_layer(blobs, x, idx, w)
    assert T.rel_l2(outs[1].cpu().numpy(), ref) <= 1e-3


def test_a_token_gets_the_same_bits_alone_and_in_a_batch():
    """Decode rows are independent: a token's output from a one-token call (split K) equals its
    row inside a 32-token call (no split)."""
    blobs, x, idx, w = _batched(2048, 768, 128, 64, 8, 32, seed=37)
    table = pk.ExpertTable(blobs)
    batch = vb.moe_forward(x, idx, w, table, path=vb.PATH_DECODE)
    for t in (0, 5, 31):
        one = vb.moe_forward(x[t:t + 1], idx[t:t + 1], w[t:t + 1], table, path=vb.PATH_DECODE)
        assert torch.equal(one[0], batch[t]), f"token {t}"


def test_new_call_fields_refuse_bad_values():
    """k_splits must be 0, 1, 2, 4 or 8 and divide hidden / 128; shared_last needs the layer's
    own combine and an act-dtype result."""
    blobs, x, idx, w = _batched(1024, 512, 128, 8, 2, 4, seed=41)
    table = pk.ExpertTable(blobs)
    with pytest.raises(RuntimeError, match="k_splits"):
        vb.moe_forward(x, idx, w, table, path=vb.PATH_DECODE, k_splits=3)
    with pytest.raises(RuntimeError, match="k_splits"):
        vb.moe_forward(x, idx, w, table, path=vb.PATH_DECODE, k_splits=16)
    with pytest.raises(RuntimeError, match="contrib"):
        vb.moe_forward(x, idx, w, table, path=vb.PATH_DECODE, shared_last=True,
                       contrib=torch.empty(8, 1024, device="cuda"))
    with pytest.raises(RuntimeError, match="activation dtype"):
        vb.moe_forward(x, idx, w, table, path=vb.PATH_DECODE, shared_last=True,
                       result=torch.empty(4, 1024, device="cuda"))
    # hidden 1024 has 8 stages of 128: 8 splits of one stage each are accepted and exact
    assert torch.equal(vb.moe_forward(x, idx, w, table, path=vb.PATH_DECODE, k_splits=8),
                       vb.moe_forward(x, idx, w, table, path=vb.PATH_DECODE, k_splits=1))


def test_a_workspace_sized_for_a_large_batch_serves_a_split_call():
    """The split-K partials of a call with few units per warp (20 tokens, top-1, 2 experts) may not
    fit a workspace sized for 128 tokens: the call then runs unsplit, with the same bits."""
    blobs, x, idx, w = _batched(2048, 768, 128, 2, 1, 128, seed=43)
    table = pk.ExpertTable(blobs)
    ws = torch.empty(pk.moe_workspace_bytes(table, 128, 1), dtype=torch.uint8, device="cuda")
    assert pk.moe_workspace_bytes(table, 20, 1) > ws.numel()      # the split needs more here
    got = vb.moe_forward(x[:20], idx[:20], w[:20], table, path=vb.PATH_DECODE, workspace=ws)
    assert torch.equal(got, vb.moe_forward(x[:20], idx[:20], w[:20], table, path=vb.PATH_DECODE))


@pytest.mark.parametrize("zeros,act", [(False, torch.bfloat16), (True, torch.bfloat16), (False, torch.float16)],
                         ids=["symmetric-bf16", "zero-points-bf16", "symmetric-fp16"])
def test_the_three_decode_decompositions_agree_bit_for_bit(zeros, act):
    """Over 64 experts at top-8: two tokens (16 routed rows) take the few-row kernels, five tokens
    (40 rows) the pass-per-CTA kernels, nine tokens (72 rows) the warp-unit kernels.  A token's
    result does not depend on the other tokens of its batch, so the shared tokens' h,
    contributions and combined rows agree bit for bit across the three."""
    blobs, x, idx, w = _batched(2048, 768, 128, 64, 8, 9, seed=47, zeros=zeros, act=act)
    table = pk.ExpertTable(blobs)
    runs = {}
    for t in (2, 5, 9):
        h = torch.empty(t * 8, 768, dtype=act, device="cuda")
        out = vb.moe_forward(x[:t], idx[:t], w[:t], table, path=vb.PATH_DECODE, h_out=h)
        c = torch.empty(t * 8, 2048, device="cuda")
        vb.moe_forward(x[:t], idx[:t], w[:t], table, path=vb.PATH_DECODE, contrib=c)
        runs[t] = (out, h, c)
    for a, b in ((2, 5), (2, 9), (5, 9)):
        assert torch.equal(runs[a][0], runs[b][0][:a]), (a, b)
        assert torch.equal(runs[a][1], runs[b][1][:a * 8]), (a, b)
        assert torch.equal(runs[a][2], runs[b][2][:a * 8]), (a, b)


def test_few_row_calls_drop_foreign_and_missing_ids_like_the_planned_path():
    """Global ids with expert_base (one expert-parallel rank's range) and -1 slots: rows outside
    the table add nothing, on the few-row and the pass-per-CTA kernels alike."""
    blobs, x, idx, w = _batched(2048, 768, 128, 64, 8, 3, seed=53)
    table = pk.ExpertTable(blobs)
    gid = idx + 16                                   # this table holds experts [16, 80)
    gid[0, 1] = -1
    gid[1, 3] = 3                                    # another rank's expert
    gid[2, 5] = 90
    out3 = vb.moe_forward(x, gid, w, table, path=vb.PATH_DECODE, expert_base=16)
    out2 = vb.moe_forward(x[:2], gid[:2], w[:2], table, path=vb.PATH_DECODE, expert_base=16)
    assert torch.equal(out2, out3[:2])
    keep = (gid[:2] >= 16) & (gid[:2] < 80)
    ref = T.oracle_layer(blobs, x[:2], torch.where(keep, gid[:2] - 16, torch.zeros_like(gid[:2])),
                         torch.where(keep, w[:2], torch.zeros_like(w[:2])))
    assert T.rel_l2(out2.cpu().numpy(), ref) <= 1e-3


