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
@pytest.mark.parametrize("batch", [1, 2, 5, 8, 9, 16])
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


@pytest.mark.parametrize("kind", ["fp8", "fp4"])
@pytest.mark.parametrize("batch", [1, 3, 8])
def test_activations_scaled_by_a_power_of_two_scale_the_output_exactly(kind, batch):
    """Batches of up to 8 tokens stage NVFP4 activations as f16 scaled per token and warp range by
    a power of two; scaling x by 2^100 or 2^-100 (and zeroing one token and a K range) must scale
    the bf16 result by exactly that factor, as it does for the bf16 products."""
    gen = torch.Generator().manual_seed(11 + batch)
    n, k = 512, 8192
    w, s = (_fp8 if kind == "fp8" else _fp4)(n, k, gen)
    x = torch.randn(batch, k, generator=gen).to(torch.bfloat16)
    x[:, 1024:2048] = 0
    if batch > 1:
        x[1] = 0
    fn = vb.fp8_gemv if kind == "fp8" else vb.fp4_gemv
    w, s = w.cuda(), s.cuda()
    base = fn(x.cuda(), w, s)
    for e in (100, -100, 60):
        got = fn((x.float() * 2.0 ** e).to(torch.bfloat16).cuda(), w, s)
        assert torch.equal(got, (base.float() * 2.0 ** e).to(torch.bfloat16)), e
    if batch > 1:
        assert not base[1].any()
    ref = (O.fp_gemv("fp8", T.to_np(w.cpu()), s.cpu().numpy(), 2, T.to_np(x)) if kind == "fp8"
           else O.fp_gemv("fp4", w.cpu().numpy(), s.cpu().numpy(), 3, T.to_np(x), gs=16))
    g, r = T.f32(T.to_np(base)), T.f32(ref)
    assert T.rel_l2(g, r) <= 1e-3 and T.max_abs_over_rms(g, r) <= 2e-2


@pytest.mark.parametrize("gs", [32, 8])
def test_fp4_other_group_sizes_match_the_oracle(gs):
    """Group 32 runs the cluster-split kernel; group 8 (not whole 16-code halves) the whole-K one."""
    gen = torch.Generator().manual_seed(gs)
    n, k = 256, 4096
    w = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, generator=gen)
    s = torch.randint(0x28, 0x48, (n, k // gs), dtype=torch.uint8, generator=gen)
    x = torch.randn(1, k, generator=gen).to(torch.bfloat16)
    got = vb.fp4_gemv(x.cuda(), w.cuda(), s.cuda())
    ref = O.fp_gemv("fp4", w.numpy(), s.numpy(), 3, T.to_np(x), gs=gs)
    g, r = T.f32(T.to_np(got)), T.f32(ref)
    assert T.rel_l2(g, r) <= 1e-3 and T.max_abs_over_rms(g, r) <= 2e-2


def test_fp8_bf16_block_scales_and_fp4_at_the_cfg4_shape_at_batch_1():
    gen = torch.Generator().manual_seed(17)
    w, s = _fp8(4096, 14336, gen)
    x = torch.randn(1, 14336, generator=gen).to(torch.bfloat16)
    sb = s.to(torch.bfloat16)
    got = vb.fp8_gemv(x.cuda(), w.cuda(), sb.cuda()).float()
    ref = x.cuda().float() @ vb.dequantize_block_scaled(w.cuda(), sb.cuda()).float().T
    assert T.rel_l2(got.cpu().numpy(), ref.cpu().numpy()) <= 4e-3
    w4, s4 = _fp4(4096, 14336, gen)
    got = vb.fp4_gemv(x.cuda(), w4.cuda(), s4.cuda()).float()
    ref = x.cuda().float() @ vb.dequantize_fp4_block_scaled(w4.cuda(), s4.cuda()).float().T
    assert T.rel_l2(got.cpu().numpy(), ref.cpu().numpy()) <= 4e-3
