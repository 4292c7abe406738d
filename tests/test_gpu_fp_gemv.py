"""GPU: FP8 / FP4 dequant fused into a decode GEMV (batch 1 and 16, the configuration-4 shapes),
against the oracle's double-summed product of the same dequantised weights."""
import numpy as np
import pytest
import torch

import vaayu_b200 as vb
from oracle import oracle as O
from tests import helpers as T

pytestmark = pytest.mark.gpu


def _fp8(n, k, gen):
    w = torch.randn(n, k, generator=gen).to(torch.float8_e4m3fn)
    s = torch.rand(n // 128, k // 128, generator=gen) * 0.02 + 1e-3
    return w, s


def _fp4(n, k, gen):
    w = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, generator=gen)
    s = torch.randint(0x28, 0x48, (n, k // 16), dtype=torch.uint8, generator=gen)
    return w, s


@pytest.mark.parametrize("kind", ["fp8", "fp4"])
@pytest.mark.parametrize("batch", [1, 16])
def test_gemv_matches_the_oracle(kind, batch):
    gen = torch.Generator().manual_seed(batch)
    n, k = 1024, 4096
    w, s = (_fp8 if kind == "fp8" else _fp4)(n, k, gen)
    x = torch.randn(batch, k, generator=gen).to(torch.bfloat16)
    if kind == "fp8":
        got = vb.fp8_gemv(x.cuda(), w.cuda(), s.cuda())
        ref = O.fp_gemv("fp8", T.to_np(w), s.numpy(), 2, T.to_np(x))
    else:
        got = vb.fp4_gemv(x.cuda(), w.cuda(), s.cuda())
        ref = O.fp_gemv("fp4", w.numpy(), s.numpy(), 3, T.to_np(x), gs=16)
    g, r = T.f32(T.to_np(got)), T.f32(ref)
    assert (T.to_np(got) == ref).mean() >= 0.99
    assert T.rel_l2(g, r) <= 1e-3 and T.max_abs_over_rms(g, r) <= 2e-2


def test_gemv_at_the_cfg4_shape():
    gen = torch.Generator().manual_seed(7)
    w, s = _fp8(4096, 14336, gen)
    x = torch.randn(16, 14336, generator=gen).to(torch.bfloat16)
    got = vb.fp8_gemv(x.cuda(), w.cuda(), s.cuda()).float()
    deq = vb.dequantize_block_scaled(w.cuda(), s.cuda()).float()
    ref = x.cuda().float() @ deq.T
    assert T.rel_l2(got.cpu().numpy(), ref.cpu().numpy()) <= 4e-3


def test_gemv_rejects_a_batch_over_16():
    gen = torch.Generator().manual_seed(1)
    w, s = _fp8(256, 1024, gen)
    with pytest.raises(NotImplementedError):
        vb.fp8_gemv(torch.zeros(17, 1024, dtype=torch.bfloat16, device="cuda"), w.cuda(), s.cuda())
