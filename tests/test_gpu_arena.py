"""GPU: layers whose experts live in an `ExpertArena` (one slab of fixed expert slots, filled from
host blobs or a checkpoint on the caller's stream) give the results of the same layer over a
blob `ExpertTable`, bit for bit, through evictions and reloads between calls (the reference's
VRAM expert tier and miss upload, vaayu/persist/expert_cache.py:813, vaayu/moe_patch.py:2829-2896)."""
import pytest
import torch

import vaayu_b200 as vb
from tests import helpers as T
from vaayu_b200 import checkpoint as ck
from vaayu_b200 import synthetic

pytestmark = pytest.mark.gpu

HID, INTER = 1024, 512


def _host_arena(blobs_cpu, capacity):
    b0 = blobs_cpu[0]
    return vb.ExpertArena(b0["geom"], b0["flat"]["scale"].dtype, "zero" in b0["flat"], len(blobs_cpu),
                          capacity, lambda e: blobs_cpu[e])


def _routing(T_, E, K, seed, experts=None):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(T_, HID, generator=g) * 0.5).to(torch.bfloat16).cuda()
    pool = torch.arange(E) if experts is None else torch.tensor(experts)
    logits = torch.randn(T_, len(pool), generator=g)
    w, j = torch.topk(logits.softmax(-1), K, -1)
    return x, pool[j].cuda(), (w / w.sum(-1, keepdim=True)).cuda()


@pytest.mark.parametrize("zeros", [False, True], ids=["symmetric", "zero-points"])
@pytest.mark.parametrize("tokens,path", [(8, vb.PATH_DECODE), (300, vb.PATH_PREFILL)], ids=["decode", "prefill"])
def test_an_arena_layer_equals_the_blob_table_layer(tokens, path, zeros):
    cpu = T.make_blobs(HID, INTER, 16, gs=128, seed=3, zeros=zeros, device="cpu")
    gpu = T.make_blobs(HID, INTER, 16, gs=128, seed=3, zeros=zeros)
    arena = _host_arena(cpu, 16)
    arena.ensure(range(16))
    x, idx, w = _routing(tokens, 16, 4, seed=tokens)
    got = vb.moe_forward(x, idx, w, arena, path=path, check=True)
    ref = vb.moe_forward(x, idx, w, vb.ExpertTable(gpu), path=path, check=True)
    assert torch.equal(got, ref)


def test_evictions_and_reloads_between_calls_keep_every_result():
    """Six slots for sixteen experts: each call routes at most four, so the sequence keeps
    evicting and reloading.  No call waits for the one before it; the results are compared only
    after the whole sequence has run, so a slot overwritten while an earlier call still read it
    would show."""
    cpu = T.make_blobs(HID, INTER, 16, gs=128, seed=8, device="cpu")
    table = vb.ExpertTable(T.make_blobs(HID, INTER, 16, gs=128, seed=8))
    arena = _host_arena(cpu, 6)
    got, ref = [], []
    for step in range(16):
        g = torch.Generator().manual_seed(100 + step)
        pick = torch.randperm(16, generator=g)[:4].tolist()
        x, idx, w = _routing(2, 16, 2, seed=step, experts=pick)
        arena.ensure(pick)
        got.append(vb.moe_forward(x, idx, w, arena, path=vb.PATH_DECODE))
        ref.append(vb.moe_forward(x, idx, w, table, path=vb.PATH_DECODE))
    torch.cuda.synchronize()
    assert arena.stats["evictions"] > 0
    assert arena.stats["misses"] > 16            # some experts came back after an eviction
    for s, (a, b) in enumerate(zip(got, ref)):
        assert torch.equal(a, b), s


def test_an_expert_parallel_rank_loads_its_range_from_safetensors(tmp_path):
    """Rank 1 of 2 over an 8-expert layer: experts [4, 8) read from the file into its arena; global
    routing ids with expert_base 4 give the rank's partial sums of the blob table over the same
    range (other ranks' slots dropped)."""
    g = torch.Generator().manual_seed(41)
    tensors = {}
    for e in range(8):
        by_role = synthetic.make_expert(HID, INTER, g, group=128)
        for role, seg in (("gate", "gate_proj"), ("down", "down_proj"), ("up", "up_proj")):
            for comp, t in by_role[role].items():
                tensors[f"model.layers.5.mlp.experts.{e}.{seg}.{comp}"] = t
    ck.write_safetensors(str(tmp_path / "m.safetensors"), tensors)
    cp = ck.Checkpoint(str(tmp_path / "m.safetensors"))
    try:
        arena = vb.ExpertArena.from_checkpoint(cp, "model.layers.5.mlp", capacity=4, experts=range(4, 8))
        assert arena.resident == [0, 1, 2, 3] and arena.stats["misses"] == 4
        table = cp.layer_table("model.layers.5.mlp", experts=range(4, 8))
        x, idx, w = _routing(6, 8, 2, seed=9)
        got = vb.moe_forward(x, idx, w, arena, path=vb.PATH_DECODE, expert_base=4)
        ref = vb.moe_forward(x, idx, w, table, path=vb.PATH_DECODE, expert_base=4)
        assert torch.equal(got, ref)
        small = vb.ExpertArena.from_checkpoint(cp, "model.layers.5.mlp", capacity=2, experts=range(4, 8),
                                               preload=False)
        for t in range(6):                       # one token at a time: two local experts per call
            local = [int(e) - 4 for e in idx[t].tolist() if e >= 4]
            small.ensure(local)
            one = vb.moe_forward(x[t:t + 1], idx[t:t + 1], w[t:t + 1], small, path=vb.PATH_DECODE, expert_base=4)
            assert torch.equal(one, ref[t:t + 1]), t
    finally:
        cp.close()
