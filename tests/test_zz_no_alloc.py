"""GPU: `vy_moe_decode_static`, the decode entry point for callers that cannot allocate device
memory (a binding that is only handed pointers, an engine with no memory left to give, code that
must not allocate while it runs).  It takes its scratch from an array built into the library
instead of a caller workspace; its results must equal `vy_moe_decode`'s, call after call, because
both run the same kernels.

This file is collected last on purpose: if it fails, a run that stops at the first failure has
already run every other test.  It passes alone in a fresh process and after the other tests."""
import ctypes

import pytest
import torch

from tests import helpers as T
from vaayu_b200 import _lib
from vaayu_b200 import packed_expert_kernels as pk

pytestmark = pytest.mark.gpu


def _static_call(table, x, idx, w, out):
    c = pk._make_call(table.geom_s, x, x.shape[0], idx.shape[1], table.n_experts,
                      table.table.data_ptr(), idx.data_ptr(), _lib.I64, w, w.stride(0), w.stride(1),
                      None, out, None, None)
    return _lib.lib().vy_moe_decode_static(ctypes.byref(c), _lib.stream_of(x.device))


def test_static_scratch_decode_equals_the_workspace_entry_point_on_consecutive_calls():
    blobs = T.make_blobs(2048, 768, 32, gs=128, seed=21)
    table = pk.ExpertTable(blobs)
    g = torch.Generator().manual_seed(3)
    for tokens in (8, 32):                                   # two calls in a row
        x = torch.randn(tokens, 2048, generator=g).to(torch.bfloat16).cuda()
        w, idx = torch.topk(torch.randn(tokens, 32, generator=g).softmax(-1), 8, -1)
        w, idx = (w / w.sum(-1, keepdim=True)).cuda(), idx.cuda()
        ref = pk.moe_forward(x, idx, w, table, path=pk.PATH_DECODE)
        out = torch.full_like(ref, float("nan"))
        _lib.check(_static_call(table, x, idx, w, out), "vy_moe_decode_static")
        torch.cuda.synchronize()
        assert T.rel_l2(out.cpu().numpy(), ref.cpu().numpy()) <= 1e-3
        assert torch.equal(out, ref)


def test_a_call_larger_than_the_static_scratch_is_rejected():
    blobs = T.make_blobs(2048, 768, 4, gs=128, seed=22)
    table = pk.ExpertTable(blobs)
    tokens = 1024                                            # ~> 8 MiB of contributions alone
    x = torch.zeros(tokens, 2048, dtype=torch.bfloat16, device="cuda")
    idx = torch.zeros(tokens, 4, dtype=torch.long, device="cuda")
    w = torch.ones(tokens, 4, device="cuda")
    out = torch.empty(tokens, 2048, device="cuda")
    with pytest.raises(NotImplementedError, match="VY_DECODE_STATIC_SCRATCH_BYTES"):
        _lib.check(_static_call(table, x, idx, w, out), "vy_moe_decode_static")
