"""Host-side logic that needs no GPU: blob layout and construction, the geometry gate, the table
payloads the kernels read, and the refusal of CPU tensors (there is no CPU path)."""
import numpy as np
import pytest
import torch

import vaayu_b200 as vb
from vaayu_b200 import packed_expert_kernels as pk
from vaayu_b200 import synthetic
from vaayu_b200.moe_patch import blob_layout, build_expert_blob, zero_layout


def test_layout_walks_the_blob_streams_in_role_order():
    """The reference's own fixture (tests/test_packed_expert_kernels.py:265-270)."""
    geom = (4, 32, (("gate", 512, 2048), ("down", 2048, 512), ("up", 512, 2048)))
    lay = pk._layout(geom)
    assert lay["gate"] == (0, 0, 512, 2048)
    assert lay["down"] == (512 * 2048 * 4 // 32, 512 * 2048 // 32, 2048, 512)
    assert lay["up"] == (2 * 512 * 2048 * 4 // 32, 2 * 512 * 2048 // 32, 512, 2048)


def test_zero_layout_holds_row_packed_words():
    geom = (4, 128, (("gate", 768, 2048), ("down", 2048, 768), ("up", 768, 2048)))
    zl = zero_layout(geom)
    assert zl["gate"] == 0
    assert zl["down"] == (768 // 8) * (2048 // 128)
    assert zl["up"] == zl["down"] + (2048 // 8) * (768 // 128)


def _expert(zeros=False, hid=256, inter=128, gs=32):
    return synthetic.make_expert(hid, inter, torch.Generator().manual_seed(3), group=gs, zeros=zeros)


def test_blob_holds_only_the_flat_streams_in_role_order():
    by_role = _expert()
    blob = build_expert_blob(by_role)
    assert set(blob["flat"]) == {"packed", "scale"}
    assert blob["geom"] == (4, 32, (("gate", 128, 256), ("down", 256, 128), ("up", 128, 256)))
    assert torch.equal(blob["flat"]["packed"],
                       torch.cat([by_role[r]["weight_packed"].reshape(-1) for r in ("gate", "down", "up")]))
    assert sum(t.nbytes for t in blob["flat"].values()) == sum(
        c["weight_packed"].nbytes + c["weight_scale"].nbytes for c in by_role.values())


def test_zero_point_blob_carries_a_zero_stream():
    by_role = _expert(zeros=True)
    blob = build_expert_blob(by_role)
    assert set(blob["flat"]) == {"packed", "scale", "zero"}
    assert blob["flat"]["zero"].numel() == zero_layout(blob["geom"])["up"] + (128 // 8) * (256 // 32)


def test_blob_refuses_g_idx_by_name_and_mixed_roles():
    by_role = _expert()
    by_role["gate"]["weight_g_idx"] = torch.zeros(256, dtype=torch.int32)
    with pytest.raises(NotImplementedError, match="g_idx"):
        build_expert_blob(by_role)
    mixed = _expert()
    mixed["down"] = synthetic.make_role(256, 128, torch.Generator().manual_seed(1), group=64)
    assert build_expert_blob(mixed) is None
    assert build_expert_blob({"gate": {"weight": torch.zeros(2)}}) is None


def test_geometry_gate():
    g = (4, 128, (("gate", 768, 2048), ("down", 2048, 768), ("up", 768, 2048)))
    assert pk._unsupported(g, torch.bfloat16, torch.float16, torch.float32) is None
    assert pk._unsupported(g, torch.float16, torch.bfloat16, torch.bfloat16) is None
    assert "int4" in pk._unsupported((8,) + g[1:], torch.bfloat16, torch.float16, torch.float32)
    assert "activation" in pk._unsupported(g, torch.float32, torch.float16, torch.float32)
    assert "group" in pk._unsupported((4, 48, g[2]), torch.bfloat16, torch.float16, torch.float32)
    odd = (4, 32, (("gate", 96, 192), ("down", 192, 96), ("up", 96, 192)))
    assert "multiples" in pk._unsupported(odd, torch.bfloat16, torch.float16, torch.float32)
    not_mlp = (4, 128, (("gate", 768, 2048), ("down", 768, 2048), ("up", 768, 2048)))
    assert "gated MLP" in pk._unsupported(not_mlp, torch.bfloat16, torch.float16, torch.float32)


def test_geometry_struct_offsets_follow_the_blob_order():
    geom = (4, 128, (("gate", 768, 2048), ("down", 2048, 768), ("up", 768, 2048)))
    s = pk._geom_struct(geom, torch.float16, True)
    lay, zl = blob_layout(geom), zero_layout(geom)
    assert (s.hidden, s.inter, s.bits, s.group_size, s.scale_dtype, s.has_zero) == (2048, 768, 4, 128, 1, 1)
    assert list(s.word_off) == [lay["gate"][0], lay["up"][0], lay["down"][0]]
    assert list(s.scale_off) == [lay["gate"][1], lay["up"][1], lay["down"][1]]
    assert list(s.zero_off) == [zl["gate"], zl["up"], zl["down"]]


def test_decode_table_payload():
    blobs = [build_expert_blob(_expert()) for _ in range(3)]
    pairs = [(blobs[0], 2), (blobs[1], 0), (blobs[2], 1)]
    vals = pk._pairs_table(pairs)
    assert vals.dtype == torch.int64 and vals.numel() == 12
    assert vals[0] == blobs[0]["flat"]["packed"].data_ptr()
    assert vals[4] == blobs[1]["flat"]["scale"].data_ptr()
    assert vals[2] == 0                                   # no zero stream
    tail = vals[9:].view(torch.int32)
    assert tail[:3].tolist() == [0, 1, 2] and tail[3:].tolist() == [2, 0, 1]


def test_prefill_payload_remaps_ids_in_ascending_order_and_drops_missing_experts():
    blobs = {e: build_expert_blob(_expert()) for e in (2, 5, 9)}
    eidx = torch.tensor([[5, 2], [2, 9], [9, 7]])           # 7 has no entry
    vals, u, entries = pk._prefill_payload(eidx, blobs)
    assert u == 3 and entries == [blobs[2], blobs[5], blobs[9]]
    ids = vals[9:].view(torch.int32)[:6].tolist()
    assert ids == [1, 0, 0, 2, 2, -1]
    assert vals[3] == blobs[5]["flat"]["packed"].data_ptr()


def test_host_plan_groups_rows_by_expert():
    """The reference's host-only table test (tests/test_packed_prefill_kernels.py:404-411)."""
    eidx = torch.tensor([[5, 2], [2, 9], [9, 5]])
    order, live, counts = pk._prefill_plan(eidx)
    assert live.tolist() == [2, 5, 9] and counts.tolist() == [2, 2, 2]
    assert order.tolist() == [1, 2, 0, 5, 3, 4]


def test_cpu_tensors_are_refused_not_served():
    """No CPU path hides behind the API: a CPU call raises instead of computing."""
    by_role = _expert()
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        vb.dequantize_packed_weight(by_role["gate"], torch.bfloat16)
    blob = build_expert_blob(by_role)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        vb.dequantize_expert_blob(blob, torch.bfloat16)
    x = torch.zeros(1, 256, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        vb.packed_experts_decode(x, [(blob, 0)], torch.ones(1, 1), torch.empty(1, 256), None)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        vb.dequantize_block_scaled(torch.zeros(4, 4).to(torch.float8_e4m3fn), torch.ones(1, 1))


def test_synthetic_generator_matches_the_baseline_script_order():
    """Codes then scales per role, roles gate/down/up, then x, then the router logits."""
    g1 = torch.Generator().manual_seed(0)
    ex = synthetic.make_expert(128, 64, g1)
    g2 = torch.Generator().manual_seed(0)
    u = torch.randint(0, 16, (64, 128), dtype=torch.int32, generator=g2).view(64, 16, 8)
    p = torch.zeros(64, 16, dtype=torch.int32)
    for j in range(8):
        p |= u[:, :, j] << (4 * j)
    assert torch.equal(ex["gate"]["weight_packed"], p)
    s = (torch.rand(64, 1, generator=g2) * 0.015 + 0.005).to(torch.float16)
    assert torch.equal(ex["gate"]["weight_scale"], s)
    assert np.all(synthetic.pack_zero_points(torch.full((9, 2), 8)).numpy() != 0)
