"""GPU: failure detection without a GPU fault (the kernels' error flags and bounded waits).

A routed expert whose table entry is unusable is skipped and flagged; a device-side barrier wait
that nothing completes runs out after its limit, flags VY_FLAG_TIMEOUT and returns, and the
context stays usable.  Nothing here traps, faults or hangs a GPU: the injected failures are a bad
table entry written by the host and a barrier that is simply never completed."""
import pytest
import torch

import vaayu_b200 as vb
from tests import helpers as T
from vaayu_b200 import _lib
from vaayu_b200 import packed_expert_kernels as pk

pytestmark = pytest.mark.gpu


def _case(tokens=12, seed=21):
    blobs = T.make_blobs(1024, 512, 8, gs=128, seed=seed)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(tokens, 1024, generator=g).to(torch.bfloat16).cuda()
    w, idx = torch.topk(torch.randn(tokens, 8, generator=g).softmax(-1), 2, -1)
    return blobs, x, idx.cuda(), (w / w.sum(-1, keepdim=True)).cuda()


@pytest.mark.parametrize("path", [vb.PATH_DECODE, vb.PATH_PREFILL], ids=["decode", "prefill"])
def test_an_unusable_expert_entry_is_flagged_and_skipped(path):
    blobs, x, idx, w = _case(tokens=12 if path == vb.PATH_DECODE else 160)
    table = pk.ExpertTable(blobs)
    clean = vb.moe_forward(x, idx, w, table, path=path, check=True)
    table.table.view(-1, 3)[3, 0] = 0                 # the host corrupts expert 3's code pointer
    with pytest.raises(RuntimeError, match="unusable"):
        vb.moe_forward(x, idx, w, table, path=path, check=True)
    got = vb.moe_forward(x, idx, w, table, path=path)  # unchecked: returns, the flag stays set
    untouched = ~(idx == 3).any(dim=1)
    assert untouched.any()
    assert torch.equal(got[untouched], clean[untouched])


def test_a_barrier_wait_that_nothing_completes_runs_out_and_reports():
    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(_lib.lib().vy_selftest_bounded_wait(2, 1_000_000, flags.data_ptr(), st), "selftest")
    torch.cuda.synchronize()
    assert int(flags.item()) == 0, "a completed barrier must not report"
    _lib.check(_lib.lib().vy_selftest_bounded_wait(1, 1_000_000, flags.data_ptr(), st), "selftest")
    torch.cuda.synchronize()
    assert int(flags.item()) & pk.FLAG_TIMEOUT
    # the context is still usable: a layer call runs and is correct
    blobs, x, idx, w = _case()
    got = vb.moe_forward(x, idx, w, pk.ExpertTable(blobs), path=vb.PATH_DECODE, check=True).cpu().numpy()
    assert T.rel_l2(got, T.oracle_layer(blobs, x, idx, w)) <= 1e-3
