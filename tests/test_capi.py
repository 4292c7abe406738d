"""The C-ABI library (no GPU needed): it loads, exports every entry point include/vaayu_b200.h
declares, and the ctypes structures have the C layout (checked against gcc's own offsetof)."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from vaayu_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "vaayu_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(vy_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_expected_surface():
    names = declared_functions()
    for required in ("vy_moe_decode", "vy_moe_prefill", "vy_moe_route_permute", "vy_moe_combine",
                     "vy_dequant_flat", "vy_fp8_dequant", "vy_fp4_dequant", "vy_fp8_gemv",
                     "vy_fp4_gemv", "vy_moe_topk_softmax", "vy_moe_workspace_size"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"
    assert set(_lib.SIGNATURES) == set(declared_functions()), "ctypes signatures drifted from the header"


def test_version_and_error_plumbing_without_a_gpu():
    lib = _lib.lib()
    assert lib.vy_abi_version() == 4
    assert isinstance(lib.vy_last_error(), bytes)


def test_workspace_size_needs_no_gpu():
    g = _lib.ExpertGeom()
    g.hidden, g.inter, g.bits, g.group_size = 2048, 768, 4, 128
    c = _lib.MoeCall()
    c.geom = ctypes.pointer(g)
    c.n_tokens, c.top_k, c.n_experts = 32, 8, 128
    small = _lib.lib().vy_moe_workspace_size(ctypes.byref(c), 0)
    c.n_tokens = 64
    assert _lib.lib().vy_moe_workspace_size(ctypes.byref(c), 0) > small > 0


def test_the_split_k_choice_shows_in_the_workspace_size():
    """A decode call of at most 16 routed rows takes the few-row kernels: no split-K partials in
    its workspace, whatever k_splits says.  A larger call with few units per warp (20 tokens,
    top-1, 2 experts) shares each gate/up unit's K range among warps and its workspace holds the
    per-stage partials; k_splits = 1 turns that off."""
    g = _lib.ExpertGeom()
    g.hidden, g.inter, g.bits, g.group_size = 2048, 768, 4, 128
    c = _lib.MoeCall()
    c.geom = ctypes.pointer(g)
    c.top_k, c.n_experts = 8, 128
    size = lambda: _lib.lib().vy_moe_workspace_size(ctypes.byref(c), 0)
    c.n_tokens, c.k_splits = 1, 0
    auto1 = size()
    c.k_splits = 4
    assert size() == auto1 > 0
    c.top_k, c.n_experts, c.n_tokens, c.k_splits = 1, 2, 20, 0
    auto20 = size()
    c.k_splits = 1
    plain20 = size()
    # the partials: (20 rows / 8 per pass + 2 live experts + 1) passes x 48 tiles of 16 rows
    # x 16 stages of 128 K x 32 lanes x 8 floats
    assert auto20 - plain20 >= 5 * 48 * 16 * 32 * 8 * 4
    c.top_k, c.n_experts, c.n_tokens, c.k_splits = 8, 128, 32, 0
    auto32 = size()
    c.k_splits = 1
    assert size() == auto32


@pytest.mark.skipif(not Path("/usr/bin/gcc").exists(), reason="gcc not available")
def test_ctypes_structures_match_the_c_layout(tmp_path):
    src = tmp_path / "layout.c"
    fields = {"vy_expert_geom": [f[0] for f in _lib.ExpertGeom._fields_],
              "vy_moe_call": [f[0] for f in _lib.MoeCall._fields_]}
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void){"]
    for st, names in fields.items():
        lines.append(f'printf("{st} %zu\\n", sizeof({st}));')
        for n in names:
            lines.append(f'printf("{st}.{n} %zu\\n", offsetof({st}, {n}));')
    lines.append("return 0;}")
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-o", str(exe), str(src)], check=True)
    got = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                        check=True).stdout.splitlines())
    for st, cls in (("vy_expert_geom", _lib.ExpertGeom), ("vy_moe_call", _lib.MoeCall)):
        assert int(got[st]) == ctypes.sizeof(cls)
        for n in fields[st]:
            assert int(got[f"{st}.{n}"]) == getattr(cls, n).offset, f"{st}.{n}"
