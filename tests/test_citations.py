"""Reference citations in the boundary header, the kernels, the C++ drop-in layer, the Python bindings and the oracle
must point inside the cited reference file: every `src/<file>:<a>-<b>` (or `:<a>`) needs b <= the file's line count.

Skipped when the reference tree is not on this machine (oracle.oracle.reference_tree()).
"""

from __future__ import annotations

import re
from pathlib import Path

import pytest

from oracle.oracle import reference_tree

REPO = Path(__file__).resolve().parent.parent
CITATION = re.compile(r"((?:src|tests)/[A-Za-z0-9_/]+\.(?:cpp|h|hpp|py))((?::\d+(?:-\d+)?)(?:,\s*:?\d+(?:-\d+)?)*)")
SCANNED = ["include", "cppinf_b200/csrc", "cppinf_b200/cpp", "cppinf_b200/ops.py", "cppinf_b200/qwen3.py",
           "cppinf_b200/shard.py", "cppinf_b200/capi.py", "oracle/oracle.c", "oracle/oracle.py", "oracle/qwen3.py",
           "oracle/ref_shim", "DESIGN.md", "INTEGRATION.md"]
SUFFIXES = {".h", ".cu", ".cuh", ".cpp", ".c", ".py", ".md"}


def scanned_files():
    for entry in SCANNED:
        path = REPO / entry
        if path.is_file():
            yield path
        elif path.is_dir():
            yield from sorted(p for p in path.rglob("*") if p.is_file() and p.suffix in SUFFIXES)


def citations(text: str):
    for number, line in enumerate(text.splitlines(), 1):
        for match in CITATION.finditer(line):
            for span in re.findall(r"\d+(?:-\d+)?", match.group(2)):
                lo, _, hi = span.partition("-")
                yield number, match.group(1), int(lo), int(hi or lo)


def test_citations_point_inside_the_cited_files():
    tree = reference_tree()
    if tree is None:
        pytest.skip("reference tree not present")
    lengths: dict[str, int] = {}
    bad, seen = [], 0
    for path in scanned_files():
        for number, rel, lo, hi in citations(path.read_text(errors="ignore")):
            seen += 1
            target = tree / rel
            if rel not in lengths:
                lengths[rel] = len(target.read_text(errors="ignore").splitlines()) if target.exists() else -1
            n = lengths[rel]
            if n < 0 or lo > hi or hi > n:
                bad.append(f"{path.relative_to(REPO)}:{number}: {rel}:{lo}-{hi} (file has {n} lines)")
    assert seen > 100, f"only {seen} citations found; the scan patterns no longer match the sources"
    assert not bad, "citations outside the cited file:\n" + "\n".join(bad)


def test_citation_pattern_reads_ranges_and_lists():
    text = "see src/ops/nn_ops.cpp:140-201 and src/nn/rope.cpp:70-74, 84-88; src/a.h:9"
    assert list(citations(text)) == [(1, "src/ops/nn_ops.cpp", 140, 201), (1, "src/nn/rope.cpp", 70, 74),
                                     (1, "src/nn/rope.cpp", 84, 88), (1, "src/a.h", 9, 9)]
