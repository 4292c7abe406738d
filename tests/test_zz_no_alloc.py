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


def _static_call(table, x, idx, w, out, k_splits=0):
    c = pk._make_call(table.geom_s, x, x.shape[0], idx.shape[1], table.n_experts,
                      table.table.data_ptr(), idx.data_ptr(), _lib.I64, w, w.stride(0), w.stride(1),
                      None, out, None, None)
    c.k_splits = k_splits
    return _lib.lib().vy_moe_decode_static(ctypes.byref(c), _lib.stream_of(x.device)), c


def test_static_scratch_decode_equals_the_workspace_entry_point_on_consecutive_calls():
    """Calls of 8 and 32 tokens, then 1 and 2 tokens with the library's K split and with four
    warps sharing a unit's K range: each reuses the scratch the call before it left behind, and
    each equals `vy_moe_decode` with its own workspace, bit for bit.  The error flags of the last
    call read back through `vy_moe_error_flags` with no workspace (the static scratch's flags)."""
    blobs = T.make_blobs(2048, 768, 32, gs=128, seed=21)
    table = pk.ExpertTable(blobs)
    g = torch.Generator().manual_seed(3)
    c = None
    for tokens, k_splits in ((8, 0), (32, 0), (1, 0), (1, 4), (2, 0), (2, 4)):
        x = torch.randn(tokens, 2048, generator=g).to(torch.bfloat16).cuda()
        w, idx = torch.topk(torch.randn(tokens, 32, generator=g).softmax(-1), 8, -1)
        w, idx = (w / w.sum(-1, keepdim=True)).cuda(), idx.cuda()
        ref = pk.moe_forward(x, idx, w, table, path=pk.PATH_DECODE, k_splits=k_splits)
        out = torch.full_like(ref, float("nan"))
        rc, c = _static_call(table, x, idx, w, out, k_splits)
        _lib.check(rc, "vy_moe_decode_static")
        torch.cuda.synchronize()
        assert T.rel_l2(out.cpu().numpy(), ref.cpu().numpy()) <= 1e-3, (tokens, k_splits)
        assert torch.equal(out, ref), (tokens, k_splits)
    flags = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    _lib.check(_lib.lib().vy_moe_error_flags(ctypes.byref(c), pk.PATH_DECODE, flags.data_ptr(),
                                             _lib.stream_of(flags.device)), "vy_moe_error_flags")
    assert int(flags.item()) == 0


def test_a_call_larger_than_the_static_scratch_is_rejected():
    blobs = T.make_blobs(2048, 768, 4, gs=128, seed=22)
    table = pk.ExpertTable(blobs)
    tokens = 1024                                            # ~> 8 MiB of contributions alone
    x = torch.zeros(tokens, 2048, dtype=torch.bfloat16, device="cuda")
    idx = torch.zeros(tokens, 4, dtype=torch.long, device="cuda")
    w = torch.ones(tokens, 4, device="cuda")
    out = torch.empty(tokens, 2048, device="cuda")
    with pytest.raises(NotImplementedError, match="VY_DECODE_STATIC_SCRATCH_BYTES"):
        _lib.check(_static_call(table, x, idx, w, out)[0], "vy_moe_decode_static")
