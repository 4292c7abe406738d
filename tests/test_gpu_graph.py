"""GPU: one CUDA graph per MoE layer for one-token decode (`packed_experts_decode_graphed`, the
contract of vaayu/packed_expert_kernels.py:531-539): a recording gives the eager bits, a replay
computes the call's own experts, and every failure leaves the layer on the eager result."""
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
    for name, val in (("_GRAPHS", {}), ("_GRAPH_OFF", {}), ("_GRAPH_NOTES", set()),
                      ("_GRAPH_VERIFIED", set()), ("GRAPH_STATS", collections.Counter())):
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
    assert (pk.GRAPH_STATS["recorded"], pk.GRAPH_STATS["replays"]) == (1, 1)


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
    assert pk.GRAPH_STATS["recorded"] == 2
    assert torch.equal(got, _eager(x2, pairs, w, None, False))


def test_inputs_that_move_every_call_keep_working(fresh, caplog):
    x, pairs, w, _b = _case(*QWEN)
    xs = [x * (i + 1) for i in range(5)]
    outs = [pk.packed_experts_decode_graphed(0, xi, pairs, w, None, None, False).clone() for xi in xs]
    torch.cuda.synchronize()
    assert 0 not in pk._GRAPH_OFF and not [r for r in caplog.records if r.levelname == "WARNING"]
    assert all(torch.equal(o, _eager(xi, pairs, w, None, False)) for o, xi in zip(outs, xs))
    assert pk.GRAPH_STATS["recorded"] == 5 and pk.GRAPH_STATS["recorded_unused"] == 4


def test_a_replay_that_disagrees_refuses_the_layer(fresh, monkeypatch, caplog):
    x, pairs, w, _b = _case(*QWEN)
    want = _eager(x, pairs, w, None, False)
    real = pk._launch
    monkeypatch.setattr(pk, "_launch", lambda x, p, w, out, h_out=None: (real(x, p, w, out), out.add_(1.0)))
    got = pk.packed_experts_decode_graphed(0, x, pairs, w, None, None, False)
    assert torch.equal(got, want + 1.0), "the eager result is returned, never the graph's"
    assert "bit for bit" in pk._GRAPH_OFF.get(0, "")
    assert any(r.levelname == "WARNING" and "stays eager" in r.getMessage() for r in caplog.records)
    assert pk.packed_experts_decode_graphed(0, x, pairs, w, None, None, False) is None


def test_a_call_the_graph_cannot_take_is_left_to_the_caller(fresh):
    x, pairs, w, _b = _case(*QWEN)
    mixed = [({"dense": {}}, pairs[0][1])] + pairs[1:]
    assert pk.packed_experts_decode_graphed(0, x, mixed, w, None, None, False) is None
    assert pk.GRAPH_STATS["recorded"] == 0


def test_the_capture_allocates_only_its_static_buffers(fresh):
    x, pairs, w, _b = _case(*QWEN)
    sh = _shared(QWEN[0])
    for _ in range(4):
        _eager(x, pairs, w, sh, True)
    pk.packed_experts_decode_graphed(99, x * 3, pairs, w, sh, None, True)
    gc.collect()
    torch.cuda.synchronize()
    m0 = torch.cuda.memory_allocated()
    pk.packed_experts_decode_graphed(0, x, pairs, w, sh, None, True)
    torch.cuda.synchronize()
    g = pk._GRAPHS[0]
    static = sum(-(-t.numel() * t.element_size() // 512) * 512
                 for t in (g.table, g.scratch, g.sum, g.cast, g.with_shared))
    held = torch.cuda.memory_allocated() - m0
    # torch's caching allocator rounds a block of 10 MB or more up to a 2 MB multiple
    assert static <= held < static + (2 << 20)
    for _ in range(50):
        pk.packed_experts_decode_graphed(0, x, pairs, w, sh, None, True)
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() - m0 == held, "a replay allocates nothing"
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
        pk._GRAPH_OFF.clear()
        (gc.enable if enabled else gc.disable)()
        try:
            out = pk.packed_experts_decode_graphed(0, x * (2 if enabled else 3), pairs, w, None, None, False)
            assert gc.isenabled() == enabled
        finally:
            gc.enable()
        assert out is not None
        assert (0 in pk._GRAPH_OFF) == capture_fails


def test_an_input_the_graph_cannot_take_warns_once(fresh, caplog):
    x, pairs, w, _b = _case(*QWEN)
    w_strided = torch.cat([w, w], dim=1)[:, ::2]
    for _ in range(3):
        assert pk.packed_experts_decode_graphed(0, x, pairs, w_strided, None, None, False) is None
    warned = [r.getMessage() for r in caplog.records if r.levelname == "WARNING"]
    assert len(warned) == 1 and "run eagerly" in warned[0]
