"""The C ABI without a GPU: the library loads, exports every symbol the
header declares, its structs have the header's layout, and its host-only
functions (the routed-GEMM planner) agree with the oracle."""

from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from tsugumi_b200 import _abi
from tsugumi_b200.moe import PrefillRoutedGEMMPlanner

HEADER = Path(__file__).resolve().parent.parent / "include" / "tsugumi_cuda.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"TSG_API\s+[\w\s\*]+?\b(tsg_\w+)\s*\(", text)


def test_library_loads_and_exports_every_declared_symbol():
    lib = _abi.load()
    names = declared_functions()
    assert len(names) >= 19
    for n in names:
        assert hasattr(lib, n), n
    assert {s[0] for s in _abi.SIGNATURES} == set(names)


def test_abi_version():
    assert _abi.load().tsg_abi_version() == 1


def test_struct_layouts_match_header():
    assert C.sizeof(_abi.ExpertOffsets) == 36
    assert C.sizeof(_abi.TokenExpertPair) == 16
    assert [getattr(_abi.TokenExpertPair, f).offset
            for f in ("token", "expert", "rank", "weight_bits_and_reserved")] == [0, 4, 8, 12]
    assert C.sizeof(_abi.MoEGroup) == 12
    assert C.sizeof(_abi.MoETile) == 16
    assert C.sizeof(_abi.RoutedGemmBlock) == 16


def test_no_gpu_context_create_fails_cleanly():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    h = C.c_void_p()
    st = _abi.load().tsg_ctx_create(0, None, C.byref(h))
    assert st != 0 and not h.value


@pytest.mark.parametrize("groups,budget", [
    ([(3, 0, 40), (7, 40, 20)], 128),
    ([(0, 0, 100), (1, 100, 100)], 128),
    ([(0, 0, 300)], 128),
    ([(0, 0, 200)], 100),
    ([(i, i, 1) for i in range(16)], 512),
    ([(i, 37 * i, 37) for i in range(9)], 96),
])
def test_host_planner_matches_oracle(groups, budget):
    g = np.zeros(len(groups), O.GROUP_DTYPE)
    for i, r in enumerate(groups):
        g[i] = r
    ref = O.plan_routed_gemm(g, budget)
    got = PrefillRoutedGEMMPlanner.plan(np.array(groups, np.uint32), budget)
    assert [b["rows"] for b in got] == [b["rows"] for b in ref]
    for a, b in zip(got, ref):
        assert a["blocks"].tolist() == [list(x) for x in b["blocks"].tolist()]


def test_host_planner_reports_too_small_capacity():
    lib = _abi.load()
    g = np.array([[0, 0, 300]], np.uint32)
    blocks = np.zeros((1, 4), np.uint32)
    rows = np.zeros(1, np.uint32)
    nb, nbatch = C.c_uint32(), C.c_uint32()
    st = lib.tsg_plan_routed_gemm(g.ctypes.data_as(C.c_void_p), 1, 128, 64,
                                  blocks.ctypes.data_as(C.c_void_p), 1, C.byref(nb),
                                  rows.ctypes.data_as(C.c_void_p), rows.ctypes.data_as(C.c_void_p),
                                  rows.ctypes.data_as(C.c_void_p), 1, C.byref(nbatch))
    assert st == 1 and nb.value == 5 and nbatch.value == 3
