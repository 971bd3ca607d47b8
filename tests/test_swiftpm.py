"""The SwiftPM C target (swift/) matches the C ABI it wraps.

There is no Swift toolchain here, so the Swift side is checked as text: the
target's header is the library's header byte for byte, the module map names
it and links the library, and every C function the Swift shim calls is one
the header declares (with the reference's Swift method names kept)."""

from __future__ import annotations

import re
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
SWIFT = ROOT / "swift"
HEADER = ROOT / "include" / "tsugumi_cuda.h"


def declared_functions() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"TSG_API\s+[\w\s\*]+?\b(tsg_\w+)\s*\(", text))


def test_target_header_is_the_library_header():
    copy = SWIFT / "Sources" / "CTsugumiCUDA" / "include" / "tsugumi_cuda.h"
    assert copy.read_bytes() == HEADER.read_bytes()


def test_module_map_exposes_header_and_links_library():
    mm = (SWIFT / "Sources" / "CTsugumiCUDA" / "include" / "module.modulemap").read_text()
    assert re.search(r"module\s+CTsugumiCUDA\s*\{", mm)
    assert 'header "tsugumi_cuda.h"' in mm
    assert 'link "tsugumi_cuda"' in mm


def test_package_declares_both_targets():
    pkg = (SWIFT / "Package.swift").read_text()
    assert 'name: "CTsugumiCUDA"' in pkg
    assert 'name: "TsugumiCUDA", dependencies: ["CTsugumiCUDA"]' in pkg
    assert (SWIFT / "Sources" / "CTsugumiCUDA" / "shim.c").exists()


def test_shim_calls_only_declared_functions_and_keeps_reference_names():
    src = (SWIFT / "Sources" / "TsugumiCUDA" / "TsugumiCUDA.swift").read_text()
    types = set(re.findall(r"\}\s*(tsg_\w+)\s*;", HEADER.read_text()))
    called = set(re.findall(r"\b(tsg_[a-z_0-9]+)\(", src)) - types  # struct inits aside
    assert called, "the shim calls nothing"
    missing = called - declared_functions()
    assert not missing, f"not in tsugumi_cuda.h: {sorted(missing)}"
    for name in ("encodeRouterGemma4BF16", "encodeRouterLogitsBF16", "groupTokenExpertPairs",
                 "makeTokenExpertPairs", "encodeStreamedTiled", "encodeReduceTokenMajor",
                 "func plan(", "final class SharedExpertRuntime"):
        assert name in src, name
