"""GPU, two devices in one process: every kernel family's per-device setup (shared-memory opt-in,
occupancy figures) is done for each device it runs on, so the same call on cuda:0 and then cuda:1
gives the same bits.  Skipped with fewer than two GPUs."""
import pytest
import torch

import vaayu_b200 as vb
from tests import helpers as T
from vaayu_b200 import packed_expert_kernels as pk

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]


def _layer_on(dev, tokens, n_exp=64, seed=61):
    blobs = T.make_blobs(2048, 768, n_exp, gs=128, seed=seed, device=dev)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(tokens, 2048, generator=g).to(torch.bfloat16).to(dev)
    w, idx = torch.topk(torch.randn(tokens, n_exp, generator=g).softmax(-1), 8, -1)
    return pk.ExpertTable(blobs), x, idx.to(dev), (w / w.sum(-1, keepdim=True)).to(dev)


@pytest.mark.parametrize("tokens", [1, 5, 32, 256], ids=["few-row", "pass-per-cta", "warp-unit", "prefill"])
def test_a_layer_call_gives_the_same_bits_on_two_devices(tokens):
    outs = []
    for d in ("cuda:0", "cuda:1"):
        table, x, idx, w = _layer_on(d, tokens)
        with torch.cuda.device(d):
            outs.append(vb.moe_forward(x, idx, w, table, check=True).cpu())
    assert torch.equal(outs[0], outs[1])


def test_the_block_scaled_gemvs_give_the_same_bits_on_two_devices():
    g = torch.Generator().manual_seed(5)
    w8 = torch.randn(512, 4096, generator=g).to(torch.float8_e4m3fn)
    s8 = torch.rand(4, 32, generator=g) * 0.02 + 1e-3
    w4 = torch.randint(0, 256, (512, 2048), dtype=torch.uint8, generator=g)
    s4 = torch.randint(0x28, 0x48, (512, 256), dtype=torch.uint8, generator=g)
    x = torch.randn(1, 4096, generator=g).to(torch.bfloat16)
    res = []
    for d in ("cuda:0", "cuda:1"):
        with torch.cuda.device(d):
            res.append((vb.fp8_gemv(x.to(d), w8.to(d), s8.to(d)).cpu(),
                        vb.fp4_gemv(x.to(d), w4.to(d), s4.to(d)).cpu()))
    assert torch.equal(res[0][0], res[1][0]) and torch.equal(res[0][1], res[1][1])
