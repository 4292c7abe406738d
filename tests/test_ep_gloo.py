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


def _worker(rank, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        from oracle import oracle as O
        from tests import helpers as TH
        from vaayu_b200.ep import ExpertParallelLayer
        experts, toks = _setup()
        per = E // 2
        local = experts[rank * per:(rank + 1) * per]

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
        layer = ExpertParallelLayer(None, E, compute=compute, combine_fn=combine, hidden=H)
        x, ids, w = toks[rank]
        got = layer.forward(x, ids, w)
        ref = O.moe_layer(_geom(), experts, TH.to_np(x), O.BF16, ids.numpy(), w.numpy(), O.F32, O.F16)
        np.save(os.path.join(result_dir, f"rank{rank}.npy"),
                np.array([np.array_equal(got.numpy(), ref), float(np.abs(got.numpy() - ref).max()),
                          uneven_refused]))
    finally:
        dist.destroy_process_group()


def test_expert_parallel_equals_one_process_bit_for_bit(tmp_path):
    mp.spawn(_worker, args=(_free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        ok, err, uneven_refused = np.load(tmp_path / f"rank{r}.npy")
        assert ok, f"rank {r}: max |diff| {err}"
        assert uneven_refused, "7 experts over 2 ranks must be refused"
