"""GPU: routing on the device -- the gather/permute plan (a stable counting sort, the reference's
host argsort + bincount, vaayu/packed_expert_kernels.py:676-717), softmax top-k, the ordered
combine and the dispatch helper."""
import numpy as np
import pytest
import torch

import vaayu_b200 as vb

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tokens,top_k,n_exp", [(1, 8, 128), (32, 8, 128), (5, 3, 7),
                                                 (2048, 2, 8), (4096, 8, 256), (300, 6, 1024)])
def test_plan_is_the_stable_argsort(tokens, top_k, n_exp):
    g = torch.Generator().manual_seed(tokens + n_exp)
    ids = torch.stack([torch.randperm(n_exp, generator=g)[:top_k] for _ in range(tokens)])
    plan = vb.route_permute(ids.cuda(), n_exp)
    flat = ids.reshape(-1)
    order = torch.argsort(flat, stable=True)
    live = torch.unique(flat)
    counts = torch.bincount(flat, minlength=n_exp)[live]
    n_live = int(plan["n_live"])
    assert n_live == live.numel() and int(plan["dropped"]) == 0
    assert torch.equal(plan["order"].cpu().long(), order)
    assert torch.equal(plan["live"][:n_live].cpu().long(), live)
    ls = plan["live_start"][:n_live + 1].cpu().long()
    assert torch.equal(ls[1:] - ls[:-1], counts)
    slot_order = torch.argsort(ids, dim=1, stable=True) + (torch.arange(tokens) * top_k)[:, None]
    assert torch.equal(plan["slot_order"].cpu().long(), slot_order)


def test_plan_with_duplicate_ids_in_a_token_is_stable_by_slot():
    ids = torch.tensor([[5, 2, 5], [2, 2, 9]], device="cuda")
    plan = vb.route_permute(ids, 16)
    assert plan["order"].tolist() == [1, 3, 4, 0, 2, 5]
    assert plan["slot_order"].tolist() == [[1, 0, 2], [3, 4, 5]]


def test_out_of_range_ids_are_dropped_and_counted():
    ids = torch.tensor([[1, 40], [-1, 1]], device="cuda")
    plan = vb.route_permute(ids, 8)
    assert int(plan["dropped"]) == 2 and int(plan["n_live"]) == 1
    assert plan["order"][:2].tolist() == [0, 3]
    assert plan["slot_order"].tolist() == [[0, -1], [3, -1]]


def test_topk_softmax_matches_torch():
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(64, 128, generator=g)
    w_ref, idx_ref = torch.topk(logits.softmax(-1), 8, -1)
    w_ref = w_ref / w_ref.sum(-1, keepdim=True)
    w, idx = vb.topk_softmax(logits.cuda(), 8)
    assert torch.equal(idx.cpu(), idx_ref)
    assert torch.allclose(w.cpu(), w_ref, rtol=2e-6, atol=1e-7)


def test_route_experts_prefers_the_models_own_router():
    class Router:
        def route_tokens_to_experts(self, logits):
            return torch.zeros(logits.shape[0], 2, dtype=torch.long), torch.ones(logits.shape[0], 2)
    w, idx = vb.route_experts(Router(), torch.randn(3, 5), 2)
    assert idx.dtype == torch.long and w.shape == (3, 2)


def test_combine_sums_in_ascending_expert_id():
    """Values chosen so fp32 addition is visibly non-associative
    (tests/test_expert_accumulation_order.py:23-38)."""
    contrib = torch.tensor([[1e8], [-1e8], [1.0]], device="cuda")
    for ids in ([[7, 2, 5]], [[2, 5, 7]], [[5, 7, 2]]):
        e = torch.tensor(ids, device="cuda")
        got = vb.combine(contrib, e)
        expected = np.float32(0)
        for k in np.argsort(np.array(ids[0]), kind="stable"):
            expected = np.float32(expected + np.float32(contrib[k, 0].item()))
        assert got.item() == expected


def test_compute_expert_dispatch():
    ids = torch.tensor([[5, 2], [2, 9], [9, 5]])
    pair, starts, counts = vb.compute_expert_dispatch(ids, 12)
    assert counts[2] == counts[5] == counts[9] == 2 and sum(counts) == 6
    assert starts[5] == 2 and starts[9] == 4
    assert pair.cpu().tolist() == [[0, 1, 0, 2, 1, 2], [1, 0, 0, 1, 1, 0]]
