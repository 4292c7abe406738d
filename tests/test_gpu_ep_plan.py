"""GPU, one device: the expert-parallel dispatch plan and combine kernels (`vy_ep_dispatch_plan`,
`vy_ep_combine`) against the torch-operation restatement of the same plan that the layer uses for
CPU tensors, bit for bit, at 1-4 destination ranks (the plan is local to one GPU; the exchange
between GPUs is tested on two devices in test_gpu_ep.py)."""
import ctypes

import pytest
import torch

import vaayu_b200 as vb
from tests import helpers as T
from vaayu_b200 import _lib
from vaayu_b200.ep import ExpertParallelLayer

pytestmark = pytest.mark.gpu

E, H = 12, 256


def _inputs(tokens, k, ids_dtype, w_dtype, seed):
    g = torch.Generator().manual_seed(seed)
    wide = torch.randn(tokens, H + 64, generator=g).to(torch.bfloat16).cuda()
    x = wide[:, 16:16 + H]                                   # a strided view: rows 320 apart
    w, idx = torch.topk(torch.randn(tokens, E, generator=g).softmax(-1), k, -1)
    return x, idx.to(ids_dtype).cuda(), w.to(w_dtype).cuda()


def _layer(ranks, placement):
    """A dispatch-mode layer object whose plan addresses `ranks` destinations (no process group:
    only the local plan is exercised)."""
    layer = ExpertParallelLayer(None, E, compute=lambda *a: None, hidden=H, mode="dispatch",
                                placement=placement)
    layer.world, layer.per_rank = ranks, E // ranks
    return layer


@pytest.mark.parametrize("ranks", [1, 2, 3, 4])
@pytest.mark.parametrize("placement", ["contiguous", "interleaved"])
@pytest.mark.parametrize("ids_dtype,w_dtype", [(torch.int64, torch.float32), (torch.int32, torch.bfloat16)],
                         ids=["i64-fp32w", "i32-bf16w"])
def test_the_device_plan_equals_the_torch_restatement(ranks, placement, ids_dtype, w_dtype):
    x, idx, w = _inputs(37, 4, ids_dtype, w_dtype, seed=ranks)
    layer = _layer(ranks, placement)
    dev = layer._dispatch_buffers(37, 4, x, w)
    layer._plan_on_device(x, idx, w, dev)
    host = {n: (t.clone() if isinstance(t, torch.Tensor) else t) for n, t in dev.items()}
    layer._plan_on_host(x, idx, w, host)                     # the same plan from torch operations
    torch.cuda.synchronize()
    assert torch.equal(dev["slot"], host["slot"])
    assert torch.equal(dev["send_id"], host["send_id"])
    filled = host["send_id"] >= 0
    assert torch.equal(dev["send_w"][filled], host["send_w"][filled])
    assert torch.equal(dev["send_x"][filled], host["send_x"][filled])
    per_dest = torch.bincount(dev["slot"] // dev["cap"], minlength=ranks)
    assert torch.equal(dev["counts"].long(), per_dest)


def _plan(idx, w, x, ranks, per_rank, cap):
    n = idx.numel()
    out = dict(send_id=torch.empty(ranks * cap, dtype=torch.int32, device="cuda"),
               send_w=torch.empty(ranks * cap, device="cuda"),
               send_x=torch.empty(ranks * cap, H, dtype=x.dtype, device="cuda"),
               slot=torch.empty(n, dtype=torch.int64, device="cuda"),
               counts=torch.empty(ranks, dtype=torch.int32, device="cuda"),
               wanted=torch.empty(ranks, dtype=torch.int32, device="cuda"))
    _lib.check(_lib.lib().vy_ep_dispatch_plan(
        idx.data_ptr(), _lib.DTYPE_CODE[idx.dtype], idx.stride(0), idx.shape[0], idx.shape[1], ranks, per_rank, 0,
        w.data_ptr(), _lib.DTYPE_CODE[w.dtype], w.stride(0), w.stride(1), x.data_ptr(), _lib.DTYPE_CODE[x.dtype],
        x.stride(0), H, cap, out["send_id"].data_ptr(), out["send_w"].data_ptr(), out["send_x"].data_ptr(),
        out["slot"].data_ptr(), out["counts"].data_ptr(), out["wanted"].data_ptr(), _lib.stream_of(x.device)),
        "vy_ep_dispatch_plan")
    return out


def test_ids_outside_the_experts_and_rows_past_a_full_destination_are_dropped():
    x, idx, w = _inputs(9, 2, torch.int64, torch.float32, seed=7)
    idx[0, 0], idx[1, 1], idx[2, 0] = -1, E, E + 5             # outside [0, E)
    idx[3:, :] = 0                                             # 12 rows for rank 0's expert 0
    out = _plan(idx, w, x, 2, E // 2, 5)                       # room for 5 rows per rank
    torch.cuda.synchronize()
    slot = out["slot"].cpu()
    flat = idx.reshape(-1).cpu()
    assert (slot[(flat < 0) | (flat >= E)] == -1).all()
    kept0 = [j for j in range(flat.numel()) if 0 <= flat[j] < E // 2]
    assert slot[kept0[:5]].tolist() == [0, 1, 2, 3, 4]         # first come, in row order
    assert (slot[kept0[5:]] == -1).all()
    assert out["counts"].cpu().tolist()[0] == 5
    assert out["wanted"].cpu().tolist()[0] == len(kept0) > 5      # the overflow stays visible
    assert (out["send_id"][:5] >= 0).all()


def test_the_combine_reads_the_returned_rows_through_the_slot_map():
    """vy_ep_combine(back, slot) equals the gathered rows' ordered combine; a dropped row adds
    nothing."""
    g = torch.Generator().manual_seed(11)
    tokens, k, n_back = 23, 4, 200
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(tokens)]).cuda()
    back = torch.randn(n_back, H, generator=g).cuda()
    slot = torch.randperm(n_back, generator=g)[:tokens * k].cuda()
    slot[5] = -1
    out = torch.empty(tokens, H, device="cuda")
    _lib.check(_lib.lib().vy_ep_combine(back.data_ptr(), slot.data_ptr(), idx.data_ptr(), _lib.DTYPE_CODE[idx.dtype],
                                        0, tokens, k, H, out.data_ptr(), out.stride(0), _lib.stream_of(back.device)),
               "vy_ep_combine")
    rows = back[slot.clamp(min=0)]
    rows[5] = 0.0
    idx_dropped = idx.clone()
    idx_dropped.view(-1)[5] = -1                               # a slot with id -1 adds nothing
    assert torch.equal(out, vb.combine(rows, idx_dropped))
    # the same ids read through a row stride (every token's row padded to k + 3 ids)
    wide = torch.full((tokens, k + 3), 999, dtype=idx.dtype, device="cuda")
    wide[:, :k] = idx
    out2 = torch.empty_like(out)
    _lib.check(_lib.lib().vy_ep_combine(back.data_ptr(), slot.data_ptr(), wide.data_ptr(), _lib.DTYPE_CODE[idx.dtype],
                                        wide.stride(0), tokens, k, H, out2.data_ptr(), out2.stride(0),
                                        _lib.stream_of(back.device)), "vy_ep_combine")
    assert torch.equal(out2, out)


@pytest.mark.parametrize("path", [vb.PATH_DECODE, vb.PATH_PREFILL], ids=["decode", "prefill"])
def test_dispatch_mode_on_one_gpu_equals_the_layer(path):
    blobs = T.make_blobs(1024, 512, 16, gs=128, seed=13)
    g = torch.Generator().manual_seed(17)
    x = torch.randn(40, 1024, generator=g).to(torch.bfloat16).cuda()
    w, idx = torch.topk(torch.randn(40, 16, generator=g).softmax(-1), 4, -1)
    w, idx = (w / w.sum(-1, keepdim=True)).cuda(), idx.cuda()
    ref = vb.moe_forward(x, idx, w, vb.ExpertTable(blobs), path=path)
    got = ExpertParallelLayer(blobs, 16, mode="dispatch", path=path).forward(x, idx, w)
    assert torch.equal(got, ref)
