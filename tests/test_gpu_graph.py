"""GPU: one CUDA graph per MoE layer for one-token decode (the reference's S28 C5 path,
tests/test_packed_expert_kernels.py:301-676): capture gives the eager bits, replay rewrites only
the table, and every failure falls back to the eager result."""
import collections
import gc

import pytest
import torch

from tests import helpers as T
from vaayu_b200 import packed_expert_kernels as pk

pytestmark = pytest.mark.gpu
QWEN = (2048, 512, 32, 10)


@pytest.fixture
def fresh(monkeypatch):
    for name, val in (("_GRAPHS", {}), ("_GRAPH_REFUSED", {}), ("_GRAPH_WARNED", set()),
                      ("GRAPH_STATS", collections.Counter())):
        monkeypatch.setattr(pk, name, val)


def _case(hid, inter, gs, k, seed=0, n_blobs=None):
    blobs = T.make_blobs(hid, inter, n_blobs or k, gs=gs, seed=hid + gs)
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(1, hid, generator=g) * 0.5).to(torch.bfloat16).cuda()
    w = torch.rand(1, k, generator=g) + 0.05
    w = (w / w.sum(-1, keepdim=True)).cuda()
    return x, [(blobs[i], i) for i in range(k)], w, blobs


def _shared(hid):
    g = torch.Generator().manual_seed(5)
    return (torch.randn(1, hid, generator=g) * 0.1).to(torch.bfloat16).cuda()


def _eager(x, pairs, w, shared, tail):
    out = torch.empty(x.shape, dtype=torch.float32, device="cuda")
    pk._launch(x, pairs, w, out)
    if not tail:
        return out
    r = out.to(x.dtype)
    return r + shared.to(r.dtype) if shared is not None else r


@pytest.mark.parametrize("tail,shared", [(False, False), (True, False), (True, True)],
                         ids=["sum", "tail", "tail+shared"])
def test_the_graph_gives_the_eager_bits(fresh, tail, shared):
    x, pairs, w, _b = _case(*QWEN)
    sh = _shared(QWEN[0]) if shared else None
    want = _eager(x, pairs, w, sh, tail)
    first = pk.packed_experts_decode_graphed(0, x, pairs, w, sh, None, tail)
    assert torch.equal(first, want)
    second = pk.packed_experts_decode_graphed(0, x, pairs, w, sh, None, tail)
    torch.cuda.synchronize()
    assert torch.equal(second, want)
    assert (pk.GRAPH_STATS["captures"], pk.GRAPH_STATS["replays"]) == (1, 1)


def test_a_rewritten_table_computes_the_new_experts(fresh):
    x, _p, w, blobs = _case(*QWEN, n_blobs=20)
    a = [(blobs[i], i) for i in range(10)]
    b = [(blobs[10 + i], i) for i in range(10)]
    pk.packed_experts_decode_graphed(0, x, a, w, None, None, False)
    got = pk.packed_experts_decode_graphed(0, x, b, w, None, None, False)
    torch.cuda.synchronize()
    assert pk.GRAPH_STATS["replays"] == 1
    assert torch.equal(got, _eager(x, b, w, None, False))


def test_a_new_input_tensor_recaptures(fresh):
    x, pairs, w, _b = _case(*QWEN)
    pk.packed_experts_decode_graphed(0, x, pairs, w, None, None, False)
    x2 = x * 2
    got = pk.packed_experts_decode_graphed(0, x2, pairs, w, None, None, False)
    assert pk.GRAPH_STATS["captures"] == 2
    assert torch.equal(got, _eager(x2, pairs, w, None, False))


def test_inputs_that_move_every_call_keep_working(fresh, capsys):
    x, pairs, w, _b = _case(*QWEN)
    xs = [x * (i + 1) for i in range(5)]
    outs = [pk.packed_experts_decode_graphed(0, xi, pairs, w, None, None, False).clone() for xi in xs]
    torch.cuda.synchronize()
    assert 0 not in pk._GRAPH_REFUSED and "WARNING" not in capsys.readouterr().out
    assert all(torch.equal(o, _eager(xi, pairs, w, None, False)) for o, xi in zip(outs, xs))
    assert pk.GRAPH_STATS["captures"] == 5 and pk.GRAPH_STATS["replaced_unreplayed"] == 4


def test_a_replay_that_disagrees_refuses_the_layer(fresh, monkeypatch, capsys):
    x, pairs, w, _b = _case(*QWEN)
    want = _eager(x, pairs, w, None, False)
    real = pk._launch
    monkeypatch.setattr(pk, "_launch", lambda x, p, w, out, h_out=None: (real(x, p, w, out), out.add_(1.0)))
    got = pk.packed_experts_decode_graphed(0, x, pairs, w, None, None, False)
    assert torch.equal(got, want + 1.0), "the eager result is returned, never the graph's"
    assert "disagrees bitwise" in pk._GRAPH_REFUSED.get(0, "")
    assert "WARNING" in capsys.readouterr().out
    assert pk.packed_experts_decode_graphed(0, x, pairs, w, None, None, False) is None


def test_a_call_the_graph_cannot_take_is_left_to_the_caller(fresh):
    x, pairs, w, _b = _case(*QWEN)
    mixed = [({"dense": {}}, pairs[0][1])] + pairs[1:]
    assert pk.packed_experts_decode_graphed(0, x, mixed, w, None, None, False) is None
    assert pk.GRAPH_STATS["captures"] == 0


def test_the_capture_allocates_only_its_static_buffers(fresh):
    x, pairs, w, _b = _case(*QWEN)
    sh = _shared(QWEN[0])
    for _ in range(len(pk._TABLES._slots)):
        _eager(x, pairs, w, sh, True)
    pk.packed_experts_decode_graphed(99, x * 3, pairs, w, sh, None, True)
    gc.collect()
    torch.cuda.synchronize()
    m0 = torch.cuda.memory_allocated()
    pk.packed_experts_decode_graphed(0, x, pairs, w, sh, None, True)
    torch.cuda.synchronize()
    g = pk._GRAPHS[0]
    static = sum(-(-t.numel() * t.element_size() // 512) * 512
                 for t in (g.tbl, g.ws, g.out, g.tmp, g.result))
    assert torch.cuda.memory_allocated() - m0 == static
    for _ in range(50):
        pk.packed_experts_decode_graphed(0, x, pairs, w, sh, None, True)
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() - m0 == static
    assert pk.GRAPH_STATS["replays"] == 50
    del g
    pk._GRAPHS.pop(0)
    gc.collect()
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() == m0, "a dropped graph returns every byte"


def test_duplicate_expert_slots_through_the_graph(fresh):
    x, pairs, w, _b = _case(*QWEN)
    dup = [pairs[0]] * 3 + pairs[1:-2]
    dup = [(blob, slot) for slot, (blob, _s) in enumerate(dup)]
    w = w.clone()
    w[0, 1:3] = 0.0
    want = _eager(x, dup, w, None, False)
    pk.packed_experts_decode_graphed(0, x, dup, w, None, None, False)
    got = pk.packed_experts_decode_graphed(0, x, dup, w, None, None, False)
    torch.cuda.synchronize()
    assert pk.GRAPH_STATS["replays"] == 1 and torch.equal(got, want)


@pytest.mark.parametrize("capture_fails", [False, True], ids=["ok", "capture-fails"])
def test_a_capture_leaves_gc_as_found(fresh, monkeypatch, capture_fails):
    x, pairs, w, _b = _case(*QWEN)
    if capture_fails:
        real = pk._decode_from_table

        def boom(*a, **kw):
            if kw.get("workspace") is not None:
                raise RuntimeError("boom")
            return real(*a, **kw)
        monkeypatch.setattr(pk, "_decode_from_table", boom)
    for enabled in (False, True):
        pk._GRAPHS.clear()
        pk._GRAPH_REFUSED.clear()
        (gc.enable if enabled else gc.disable)()
        try:
            out = pk.packed_experts_decode_graphed(0, x * (2 if enabled else 3), pairs, w, None, None, False)
            assert gc.isenabled() == enabled
        finally:
            gc.enable()
        assert out is not None
        assert (0 in pk._GRAPH_REFUSED) == capture_fails


def test_an_input_the_graph_cannot_take_warns_once(fresh, capsys):
    x, pairs, w, _b = _case(*QWEN)
    w_strided = torch.cat([w, w], dim=1)[:, ::2]
    for _ in range(3):
        assert pk.packed_experts_decode_graphed(0, x, pairs, w_strided, None, None, False) is None
    out = capsys.readouterr().out
    assert out.count("WARNING") == 1 and "not used" in out
