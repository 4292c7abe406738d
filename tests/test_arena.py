"""Host bookkeeping of the expert arena (slots, LRU order, pointer-table entries), on CPU: the slab
and tables live in host memory here, so every address the kernels would read can be checked."""
import pytest
import torch

import vaayu_b200 as vb
from tests.helpers import make_blobs


def _arena(n=8, capacity=3, zeros=False):
    blobs = make_blobs(256, 128, n, gs=32, seed=5, zeros=zeros, device="cpu")
    loads = []

    def loader(e):
        loads.append(e)
        return blobs[e]
    b0 = blobs[0]
    arena = vb.ExpertArena(b0["geom"], b0["flat"]["scale"].dtype, zeros, n, capacity, loader, device="cpu")
    return arena, blobs, loads


def _check_resident(arena, blobs):
    base = arena.slab.data_ptr()
    names = ["packed", "scale"] + (["zero"] if arena.has_zero else [])
    for e in range(arena.n_experts):
        entry = arena.table[3 * e: 3 * e + 3].tolist()
        if e not in arena.resident:
            assert entry == [0, 0, 0], e
            continue
        slot = arena._slot_of[e]
        views = arena.stream_views(slot)
        for j, name in enumerate(names):
            assert entry[j] == views[name].data_ptr(), (e, name)
            assert entry[j] % 256 == 0 and base <= entry[j] < base + arena.slab.numel()
            assert torch.equal(views[name], blobs[e]["flat"][name]), (e, name)
        if not arena.has_zero:
            assert entry[2] == 0


@pytest.mark.parametrize("zeros", [False, True])
def test_slots_fill_then_evict_the_least_recently_used(zeros):
    arena, blobs, loads = _arena(zeros=zeros)
    arena.ensure([1, 0, 1])
    assert arena.resident == [0, 1] and loads == [0, 1]
    arena.ensure(torch.tensor([[2], [0]]))              # 0 hit: 1 is now the least recent
    assert arena.resident[0] == 1 and sorted(arena.resident) == [0, 1, 2] and loads == [0, 1, 2]
    _check_resident(arena, blobs)
    arena.ensure([3])                                   # evicts 1, the least recently used
    assert sorted(arena.resident) == [0, 2, 3] and loads[-1] == 3
    _check_resident(arena, blobs)
    arena.ensure([1, 2])                                # needs 2 -> evicts 0, not 2
    assert sorted(arena.resident) == [1, 2, 3] and 0 not in arena.resident
    _check_resident(arena, blobs)
    assert arena.stats["evictions"] == 2 and arena.stats["misses"] == 5
    arena.ensure([7, -1, 99])                           # out-of-range ids are ignored
    assert 7 in arena.resident
    _check_resident(arena, blobs)


def test_evict_frees_the_slot_and_clears_the_entry():
    arena, blobs, _ = _arena()
    arena.ensure([4, 5, 6])
    slot = arena._slot_of[5]
    arena.evict(5)
    assert arena.table[15:18].tolist() == [0, 0, 0]
    arena.ensure([0])
    assert arena._slot_of[0] == slot and sorted(arena.resident) == [0, 4, 6]
    _check_resident(arena, blobs)


def test_a_call_routing_more_experts_than_slots_is_refused():
    arena, _, _ = _arena(capacity=2)
    with pytest.raises(RuntimeError, match="holds 2"):
        arena.ensure([0, 1, 2])


def test_an_expert_of_another_format_is_refused():
    blobs = make_blobs(256, 128, 2, gs=32, seed=1, device="cpu")
    other = make_blobs(256, 128, 1, gs=64, seed=2, device="cpu")[0]
    arena = vb.ExpertArena(blobs[0]["geom"], torch.float16, False, 2, 2,
                           lambda e: blobs[0] if e == 0 else other, device="cpu")
    arena.ensure([0])
    with pytest.raises(NotImplementedError, match="expert 1"):
        arena.ensure([1])


def test_a_rank_range_loads_from_safetensors_into_the_slab(tmp_path):
    """`from_checkpoint` over experts [4, 8) of an 8-expert layer file: local expert i is file
    expert 4 + i, its slot holds exactly the blob the checkpoint reader builds, and a miss reads
    only that expert."""
    from vaayu_b200 import checkpoint as ck
    from vaayu_b200 import synthetic
    g = torch.Generator().manual_seed(3)
    tensors = {}
    for e in range(8):
        by_role = synthetic.make_expert(256, 128, g, group=32)
        for role, seg in (("gate", "gate_proj"), ("down", "down_proj"), ("up", "up_proj")):
            for comp, t in by_role[role].items():
                tensors[f"model.layers.1.mlp.experts.{e}.{seg}.{comp}"] = t
    ck.write_safetensors(str(tmp_path / "m.safetensors"), tensors)
    cp = ck.Checkpoint(str(tmp_path / "m.safetensors"))
    try:
        arena = vb.ExpertArena.from_checkpoint(cp, "model.layers.1.mlp", capacity=2, experts=range(4, 8),
                                               device="cpu")
        assert arena.n_experts == 4 and arena.resident == [0, 1]
        arena.ensure([3])
        assert arena.resident == [1, 3]            # expert 0 was the least recently used
        for local in arena.resident:
            want = cp.expert_blob("model.layers.1.mlp", 4 + local, device="cpu")
            got = arena.stream_views(arena._slot_of[local])
            for name in ("packed", "scale"):
                assert torch.equal(got[name], want["flat"][name]), (local, name)
    finally:
        cp.close()
