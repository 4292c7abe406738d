"""GPU: expert parallelism over NCCL on 2 GPUs -- dispatch mode equals the single-GPU layer bit
for bit; replicate mode is exactly the rank-ordered sum of per-rank partials, deterministic, and
within fp32 rounding of the single-GPU layer.  Skipped with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, result_dir):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        import vaayu_b200 as vb
        from tests import helpers as T
        from vaayu_b200.ep import ExpertParallelLayer
        dev = torch.device("cuda", rank)
        E, K, tokens = 16, 4, 12
        blobs = T.make_blobs(1024, 512, E, gs=128, seed=5, device=dev)
        g = torch.Generator().manual_seed(100 + rank)
        x = torch.randn(tokens, 1024, generator=g).to(torch.bfloat16).to(dev)
        w, idx = torch.topk(torch.randn(tokens, E, generator=g).softmax(-1), K, -1)
        w, idx = (w / w.sum(-1, keepdim=True)).to(dev), idx.to(dev)
        local = blobs[rank * E // 2:(rank + 1) * E // 2]
        table = vb.ExpertTable(blobs)
        ref = vb.moe_forward(x, idx, w, table, path=vb.PATH_DECODE)
        # dispatch mode: the same fp32 sum in the same order as one GPU
        got = ExpertParallelLayer(local, E, mode="dispatch").forward(x, idx, w)
        # replicate mode: each rank's partial (its experts' slots in ascending id), rank order
        rep = ExpertParallelLayer(local, E, mode="replicate")
        got_r = rep.forward(x, idx, w)
        again = rep.forward(x, idx, w)
        exp = None
        for q in range(2):
            lo = torch.where((idx >= q * E // 2) & (idx < (q + 1) * E // 2), idx, torch.full_like(idx, -1))
            part = vb.moe_forward(x, lo, w, table, path=vb.PATH_DECODE)
            exp = part if q == 0 else exp + part
        torch.cuda.synchronize()
        rel = float((got_r - ref).abs().max() / ref.pow(2).mean().sqrt())
        np.save(os.path.join(result_dir, f"rank{rank}.npy"),
                np.array([torch.equal(got, ref), float((got - ref).abs().max()), torch.equal(got_r, exp),
                          torch.equal(got_r, again), rel]))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_expert_parallel_over_nccl_equals_one_gpu(tmp_path):
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(_free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        ok, err, rep_exact, rep_repeat, rep_rel = np.load(tmp_path / f"rank{r}.npy")
        assert ok, f"dispatch mode, rank {r}: max |diff| {err}"
        assert rep_exact, f"replicate mode, rank {r}: not the rank-ordered sum of per-rank partials"
        assert rep_repeat, f"replicate mode, rank {r}: two calls differ"
        assert rep_rel < 1e-5, f"replicate mode, rank {r}: {rep_rel} of RMS from one GPU"
