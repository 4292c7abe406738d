"""Expert parallelism's host logic on CPU: two `gloo` ranks, the oracle standing in for the GPU
kernels as each rank's per-row compute.  Dispatch, the variable all-to-all, the return path and
the combine in ascending GLOBAL expert id must give exactly the single-process layer."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

H, I, E, K, T = 256, 128, 8, 3, 5


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup():
    from vaayu_b200 import synthetic
    from tests import helpers as TH
    g = torch.Generator().manual_seed(123)
    experts = [TH.expert_from_components(synthetic.make_expert(H, I, g, group=32)) for _ in range(E)]
    toks = []
    for r in range(2):
        gr = torch.Generator().manual_seed(7 + r)
        x = torch.randn(T, H, generator=gr).to(torch.bfloat16)
        ids = torch.stack([torch.randperm(E, generator=gr)[:K] for _ in range(T)])
        ids[0, 1] = ids[0, 0] if r == 0 else ids[0, 1]       # a duplicated expert in one token
        w = torch.rand(T, K, generator=gr) + 0.05
        toks.append((x, ids, w / w.sum(-1, keepdim=True)))
    return experts, toks


def _geom():
    return (4, 32, (("gate", I, H), ("down", H, I), ("up", I, H)))


def _worker(rank, port, result_dir, placement="contiguous"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        from oracle import oracle as O
        from tests import helpers as TH
        from vaayu_b200.ep import ExpertParallelLayer
        experts, toks = _setup()
        per = E // 2
        local = experts[rank * per:(rank + 1) * per] if placement == "contiguous" else experts[rank::2]

        def compute(x_rows, local_ids, w_rows):
            if x_rows.shape[0] == 0:
                return torch.zeros(0, H)
            _o, y = O.moe_layer(_geom(), local, TH.to_np(x_rows), O.BF16, local_ids.numpy().astype(np.int64),
                                w_rows.reshape(-1).numpy(), O.F32, O.F16, want_y=True)
            return torch.from_numpy(y)

        def combine(rows, ids):
            rows, ids = rows.numpy(), ids.numpy()
            out = np.zeros((ids.shape[0], H), np.float32)
            for t in range(ids.shape[0]):
                for k in np.argsort(ids[t], kind="stable"):
                    out[t] = (out[t] + rows[t * K + k]).astype(np.float32)
            return torch.from_numpy(out)

        try:
            ExpertParallelLayer(None, E - 1, compute=compute, hidden=H)
            uneven_refused = False
        except ValueError:
            uneven_refused = True
        layer = ExpertParallelLayer(None, E, compute=compute, combine_fn=combine, hidden=H, mode="dispatch",
                                    placement=placement)
        x, ids, w = toks[rank]
        got = layer.forward(x, ids, w)
        ref = O.moe_layer(_geom(), experts, TH.to_np(x), O.BF16, ids.numpy(), w.numpy(), O.F32, O.F16)
        np.save(os.path.join(result_dir, f"rank{rank}.npy"),
                np.array([np.array_equal(got.numpy(), ref), float(np.abs(got.numpy() - ref).max()),
                          uneven_refused]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("placement", ["contiguous", "interleaved"])
def test_dispatch_mode_equals_one_process_bit_for_bit(tmp_path, placement):
    mp.spawn(_worker, args=(_free_port(), str(tmp_path), placement), nprocs=2, join=True)
    for r in range(2):
        ok, err, uneven_refused = np.load(tmp_path / f"rank{r}.npy")
        assert ok, f"rank {r}: max |diff| {err}"
        assert uneven_refused, "7 experts over 2 ranks must be refused"


# ── replicate mode: all-gathered tokens, per-rank partial sums, rank-ordered combine ──────────

def _partials(local_experts, xa, local, wa):
    """Per-token fp32 sum of the local slots' contributions, ascending local expert id then slot."""
    from oracle import oracle as O
    from tests import helpers as TH
    local = np.asarray(local)
    out = np.zeros((local.shape[0], H), np.float32)
    rows = [(t, k) for t in range(local.shape[0]) for k in range(local.shape[1]) if local[t, k] >= 0]
    if not rows:
        return out
    xr = TH.to_np(xa)[[t for t, _ in rows]]
    ids = np.array([[local[t, k]] for t, k in rows], np.int64)
    ws = np.array([float(wa[t, k]) for t, k in rows], np.float32)
    _o, y = O.moe_layer(_geom(), local_experts, xr, O.BF16, ids, ws, O.F32, O.F16, want_y=True)
    by_tok = {}
    for i, (t, k) in enumerate(rows):
        by_tok.setdefault(t, []).append((int(local[t, k]), k, i))
    for t, lst in by_tok.items():
        for _e, _k, i in sorted(lst):
            out[t] = (out[t] + y[i]).astype(np.float32)
    return out


def _replicate_worker(rank, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        from oracle import oracle as O
        from tests import helpers as TH
        from vaayu_b200.ep import ExpertParallelLayer
        experts, toks = _setup()
        per = E // 2
        local_experts = experts[rank * per:(rank + 1) * per]
        layer = ExpertParallelLayer(None, E, hidden=H, mode="replicate",
                                    layer_fn=lambda xa, lo, wa: torch.from_numpy(_partials(local_experts, xa, lo, wa)))
        x, ids, w = toks[rank]
        got = layer.forward(x, ids, w).numpy()
        again = layer.forward(x, ids, w).numpy()
        # the expectation in one process: each rank's partial over this rank's tokens, summed in
        # rank order
        exp = np.zeros((T, H), np.float32)
        for q in range(2):
            lo = ids.numpy() - q * per
            lo = np.where((lo >= 0) & (lo < per), lo, -1)
            part = _partials(experts[q * per:(q + 1) * per], x, lo, w.numpy())
            exp = part.copy() if q == 0 else (exp + part).astype(np.float32)
        full = O.moe_layer(_geom(), experts, TH.to_np(x), O.BF16, ids.numpy(), w.numpy(), O.F32, O.F16)
        np.save(os.path.join(result_dir, f"rep{rank}.npy"),
                np.array([np.array_equal(got, exp), np.array_equal(got, again),
                          float(np.abs(got - full).max() / (np.sqrt(np.mean(full ** 2)) + 1e-30))]))
    finally:
        dist.destroy_process_group()


def test_replicate_mode_is_the_rank_ordered_sum_of_per_rank_partials(tmp_path):
    """Exact: (rank 0's slots summed in ascending id) + (rank 1's ...), deterministic across
    calls, and within fp32 rounding of the single-process layer."""
    mp.spawn(_replicate_worker, args=(_free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        exact, repeat, rel = np.load(tmp_path / f"rep{r}.npy")
        assert exact, f"rank {r}: not the rank-ordered partial sum"
        assert repeat, f"rank {r}: two calls differ"
        assert rel < 1e-5, f"rank {r}: {rel} of RMS from the single-process layer"


# ── failure detection: a rank that never joins the exchange ──────────────────────────────────

def _dropped_worker(rank, port, result_dir):
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=3))
    try:
        from vaayu_b200.ep import ExpertParallelLayer
        _experts, toks = _setup()
        if rank == 1:
            time.sleep(6)          # never reaches the collective before rank 0's timeout
            return
        layer = ExpertParallelLayer(None, E, hidden=H, mode="replicate",
                                    layer_fn=lambda xa, lo, wa: torch.zeros(xa.shape[0], H))
        x, ids, w = toks[0]
        t0 = time.time()
        try:
            layer.forward(x, ids, w)
            outcome = 0.0
        except Exception:      # noqa: BLE001 -- the timeout surfaces as an exception, not a hang
            outcome = 1.0
        np.save(os.path.join(result_dir, "dropped.npy"), np.array([outcome, time.time() - t0]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:      # noqa: BLE001
            pass


def test_a_rank_that_never_joins_makes_the_others_raise_not_hang(tmp_path):
    mp.spawn(_dropped_worker, args=(_free_port(), str(tmp_path)), nprocs=2, join=True)
    raised, seconds = np.load(tmp_path / "dropped.npy")
    assert raised == 1.0, "the exchange with a missing rank must raise"
    assert seconds < 30


# ── the dispatch plan itself (one process, no exchange) ───────────────────────────────────────

@pytest.mark.parametrize("placement", ["contiguous", "interleaved"])
def test_the_dispatch_plan_files_rows_stably_by_destination(placement):
    """Every (token, slot) row lands in its expert's rank's slot range, ranked among that rank's
    rows in row order; empty slots carry id -1.  (The library's device plan is held to this same
    plan bit for bit in test_gpu_ep_plan.py.)"""
    from vaayu_b200.ep import ExpertParallelLayer
    n_exp, ranks, tokens, k, hid = 12, 3, 10, 4, 8
    layer = ExpertParallelLayer(None, n_exp, compute=lambda *a: None, hidden=hid, mode="dispatch",
                                placement=placement)
    layer.world, layer.per_rank = ranks, n_exp // ranks
    g = torch.Generator().manual_seed(5)
    ids = torch.stack([torch.randperm(n_exp, generator=g)[:k] for _ in range(tokens)])
    w = torch.rand(tokens, k, generator=g)
    x = torch.randn(tokens, hid, generator=g).to(torch.bfloat16)
    b = layer._dispatch_buffers(tokens, k, x, w)
    layer._plan_on_host(x, ids, w, b)
    cap = b["cap"]
    nxt = [0] * ranks
    for j, e in enumerate(ids.reshape(-1).tolist()):
        d, local = (e % ranks, e // ranks) if placement == "interleaved" else (e // (n_exp // ranks), e % (n_exp // ranks))
        slot = d * cap + nxt[d]
        nxt[d] += 1
        assert b["slot"][j] == slot
        assert b["send_id"][slot] == local
        assert b["send_w"][slot] == w.reshape(-1)[j]
        assert torch.equal(b["send_x"][slot], x[j // k])
    for d in range(ranks):
        assert (b["send_id"][d * cap + nxt[d]:(d + 1) * cap] == -1).all()


# ── dispatch capacity: a recorded bound, overflow flagged ────────────────────────────────────

def _capacity_worker(rank, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        from oracle import oracle as O
        from tests import helpers as TH
        from vaayu_b200.ep import ExpertParallelLayer
        experts, _toks = _setup()
        per = E // 2
        local = experts[rank * per:(rank + 1) * per]

        def compute(x_rows, local_ids, w_rows):
            _o, y = O.moe_layer(_geom(), local, TH.to_np(x_rows), O.BF16, local_ids.numpy().astype(np.int64),
                                w_rows.reshape(-1).numpy(), O.F32, O.F16, want_y=True)
            return torch.from_numpy(y)

        def combine(rows, ids_):
            rows, ids_ = rows.numpy(), ids_.numpy()
            out = np.zeros((ids_.shape[0], H), np.float32)
            for t in range(ids_.shape[0]):
                for k in np.argsort(ids_[t], kind="stable"):
                    out[t] = (out[t] + rows[t * K + k]).astype(np.float32)
            return torch.from_numpy(out)

        layer = ExpertParallelLayer(None, E, compute=compute, combine_fn=combine, hidden=H, mode="dispatch",
                                    capacity_margin=1.0)
        tokens = 32
        gr = torch.Generator().manual_seed(40 + rank)
        x = torch.randn(tokens, H, generator=gr).to(torch.bfloat16)
        ids = torch.stack([torch.randperm(E, generator=gr)[:K] for _ in range(tokens)])
        w = torch.rand(tokens, K, generator=gr) + 0.05
        w = w / w.sum(-1, keepdim=True)
        ref = O.moe_layer(_geom(), experts, TH.to_np(x), O.BF16, ids.numpy(), w.numpy(), O.F32, O.F16)
        first = layer.forward(x, ids, w)                          # records the bound
        cap = layer._caps[(tokens, K)]
        same = np.array_equal(first.numpy(), ref) and not layer.overflowed()
        # every row of both ranks to rank 0's experts: more rows than the recorded bound
        crowded = torch.stack([torch.tensor([0, 1, 2]) for _ in range(tokens)])
        layer.forward(x, crowded, w)
        over = layer.overflowed()
        np.save(os.path.join(result_dir, f"cap{rank}.npy"), np.array([same, cap < tokens * K, over]))
    finally:
        dist.destroy_process_group()


def test_dispatch_capacity_is_a_recorded_bound_and_an_overflow_is_flagged(tmp_path):
    mp.spawn(_capacity_worker, args=(_free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        same, bounded, over = np.load(tmp_path / f"cap{r}.npy")
        assert same, f"rank {r}: the bounded exchange must equal the one-process layer"
        assert bounded, "the recorded capacity should be below T * K for this routing"
        assert over, f"rank {r}: the crowded call overflows rank 0's slots"
