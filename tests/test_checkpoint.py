"""Host logic of the checkpoint reader: the reference's role grouping
(vaayu/moe_patch.py:527-551, 591-594; its tests tests/test_packed_expert_dequant.py:149-163 and
tests/test_moe_miss_helpers.py:31-35) and safetensors round trips at the checkpoint's bit width."""
import torch

import vaayu_b200 as vb
from vaayu_b200 import checkpoint as ck
from vaayu_b200 import synthetic

COMPONENTS = ("weight_packed", "weight_scale", "weight_shape")


def _raw(prefix="model.layers.0.mlp.experts.3", names=("gate_proj", "down_proj", "up_proj"), zeros=False,
         seed=0, hid=256, inter=128):
    g = torch.Generator().manual_seed(seed)
    by_role = synthetic.make_expert(hid, inter, g, group=32, zeros=zeros)
    raw = {}
    for role, seg in zip(("gate", "down", "up"), names):
        for comp, t in by_role[role].items():
            raw[f"{prefix}.{seg}.{comp}"] = t
    return raw, by_role


def test_grouping_maps_every_component_to_its_role():
    raw, by_role = _raw()
    groups = ck.group_packed_tensors_by_weight(raw)
    assert set(groups) == {"gate", "down", "up"}
    for role in groups:
        assert set(groups[role]) == set(by_role[role])
        for comp, t in groups[role].items():
            assert torch.equal(t, by_role[role][comp])


def test_grouping_is_empty_for_a_dense_expert():
    dense = {f"m.experts.0.{s}.weight": torch.zeros(2) for s in ("gate_proj", "down_proj", "up_proj")}
    assert all(not v for v in ck.group_packed_tensors_by_weight(dense).values())


def test_roles_complete_needs_codes_and_scales_of_every_role():
    groups = ck.group_packed_tensors_by_weight(_raw()[0])
    assert ck.packed_roles_complete(groups)
    del groups["up"]["weight_scale"]
    assert not ck.packed_roles_complete(groups)


def test_mixtral_names_group_like_the_reference():
    raw, by_role = _raw(prefix="model.layers.0.block_sparse_moe.experts.1", names=("w1", "w2", "w3"))
    groups = ck.group_packed_tensors_by_weight(raw)
    assert torch.equal(groups["down"]["weight_packed"], by_role["down"]["weight_packed"])


def test_safetensors_round_trip_builds_the_same_blobs(tmp_path):
    """A two-file checkpoint with four experts (one with zero points, one dense): each packed
    expert's blob equals `build_expert_blob` of its in-memory components, bit for bit."""
    files = [{}, {}]
    mem = {}
    for e in range(4):
        raw, by_role = _raw(prefix=f"model.layers.2.mlp.experts.{e}", zeros=(e == 1), seed=10 + e)
        if e == 3:
            raw = {k.replace("weight_packed", "weight"): torch.randn(4, 4) for k in raw if k.endswith("weight_packed")}
        else:
            mem[e] = vb.build_expert_blob(by_role)
        files[e % 2].update(raw)
    files[0]["model.layers.2.mlp.gate.weight"] = torch.randn(4, 256)
    for i, t in enumerate(files):
        ck.write_safetensors(str(tmp_path / f"model-{i:05d}.safetensors"), t)
    cp = ck.Checkpoint(str(tmp_path))
    try:
        assert cp.experts("model.layers.2.mlp") == [0, 1, 2, 3]
        for e in (0, 1, 2):
            blob = cp.expert_blob("model.layers.2.mlp", e, device="cpu")
            assert blob["geom"] == mem[e]["geom"]
            assert set(blob["flat"]) == set(mem[e]["flat"])
            for k, t in mem[e]["flat"].items():
                assert torch.equal(blob["flat"][k], t), (e, k)
        assert cp.expert_blob("model.layers.2.mlp", 3, device="cpu") is None      # dense
        assert set(cp.read_expert("model.layers.2.mlp", 0)) == {
            f"model.layers.2.mlp.experts.0.{s}.{c}" for s in ("gate_proj", "down_proj", "up_proj")
            for c in COMPONENTS}
    finally:
        cp.close()


def test_bf16_and_fp8_tensors_read_back_exactly(tmp_path):
    t = {"a": torch.randn(3, 5).to(torch.bfloat16), "b": torch.randn(7).to(torch.float8_e4m3fn),
         "c": torch.arange(6, dtype=torch.int32).reshape(2, 3)}
    ck.write_safetensors(str(tmp_path / "x.safetensors"), t, metadata={"format": "pt"})
    f = ck.SafetensorsFile(str(tmp_path / "x.safetensors"))
    try:
        for k, v in t.items():
            r = f.tensor(k)
            assert r.dtype == v.dtype and r.shape == v.shape
            assert torch.equal(r.view(torch.uint8), v.view(torch.uint8))
    finally:
        f.close()


def test_lowest_expert_and_the_install_probe_read_the_layer_file(tmp_path):
    """The engine's per-layer file `<checkpoint_path>/<layer_name>.safetensors`: the install probe
    reads its lowest-numbered expert with this package's reader (no engine loader) and builds the
    same blob as the in-memory components."""
    from types import SimpleNamespace

    from vaayu_b200 import packed_expert_kernels as pk
    tensors, mem = {}, {}
    for e in (7, 2, 5):
        raw, by_role = _raw(prefix=f"model.layers.4.mlp.experts.{e}", seed=30 + e)
        tensors.update(raw)
        mem[e] = vb.build_expert_blob(by_role)
    ck.write_safetensors(str(tmp_path / "model.layers.4.mlp.safetensors"), tensors)
    cp = ck.Checkpoint(str(tmp_path / "model.layers.4.mlp.safetensors"))
    try:
        assert cp.lowest_expert() == ("model.layers.4.mlp", 2)
    finally:
        cp.close()
    engine = SimpleNamespace(checkpoint_path=str(tmp_path))
    block = SimpleNamespace(layer_name="model.layers.4.mlp", layer_idx=4)
    blob = pk._probe_blob(engine, block, "cpu")
    assert blob["geom"] == mem[2]["geom"]
    for k, t in mem[2]["flat"].items():
        assert torch.equal(blob["flat"][k], t), k
    # the host's own probe wins; a missing layer file reads as "no blob"
    engine.packed_probe_blob = lambda b, d: mem[5]
    assert pk._probe_blob(engine, block, "cpu") is mem[5]
    assert pk._probe_blob(SimpleNamespace(checkpoint_path=str(tmp_path)),
                          SimpleNamespace(layer_name="model.layers.9.mlp"), "cpu") is None


def test_install_leaves_a_cpu_model_and_a_model_without_fused_blocks_alone():
    from types import SimpleNamespace

    from vaayu_b200 import packed_expert_kernels as pk
    cpu_model = SimpleNamespace(running_device="cpu", running_dtype=torch.bfloat16, _moe_blocks=[])
    assert pk.install_packed_expert_kernels(cpu_model) is False
    assert not hasattr(cpu_model, "_packed_moe_kernel")
    assert pk._is_silu(torch.nn.functional.silu, "cpu", torch.float32)
    assert not pk._is_silu(torch.nn.functional.gelu, "cpu", torch.float32)
    assert not pk._is_silu(None, "cpu", torch.float32)
