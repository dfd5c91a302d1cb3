"""Every reference citation in the repository (`src/...:a-b`, `include/...:n`, `tests/...`,
`convert/...`, `tools/...`) names a file of the reference tree and lines that exist in it.
Runs where the reference tree is found (LEVO_REFERENCE_ROOT, or BASELINE.json's
reference_path); skipped elsewhere."""
from __future__ import annotations

import re
import subprocess

import pytest

from conftest import ROOT, entry

CITATION = re.compile(r"((?:src|include|tests|convert|tools|docs)/[\w./+-]+\.(?:cpp|h|hpp|py|md|c|txt)):"
                      r"(\d+(?:-\d+)?(?:,\d+(?:-\d+)?)*)")
# Files that describe the reference in prose written by others, not by this repository.
SKIP = {"SURVEY.md", "VERDICT.md", "ADVICE.md", "BASELINE.md", "BASELINE.json"}


def _cited_files():
    out = subprocess.run(["git", "ls-files"], cwd=ROOT, capture_output=True, text=True).stdout.split()
    for name in sorted(set(out)):
        if name in SKIP or name.startswith(("_work/", "baseline/")):
            continue
        path = ROOT / name
        if path.suffix in (".npz", ".so", ".o", ".json", ".jsonl") or not path.is_file():
            continue
        yield name, path


def test_every_reference_citation_exists():
    ref = entry.reference_root()
    if ref is None:
        pytest.skip("reference tree not found (set LEVO_REFERENCE_ROOT)")
    bad, count = [], 0
    for name, path in _cited_files():
        for lineno, line in enumerate(path.read_text(errors="ignore").splitlines(), 1):
            for m in CITATION.finditer(line):
                count += 1
                target = ref / m.group(1)
                if not target.is_file():
                    bad.append(f"{name}:{lineno}: {m.group(1)} does not exist")
                    continue
                n_lines = len(target.read_text(errors="ignore").splitlines())
                for part in m.group(2).split(","):
                    lo, _, hi = part.partition("-")
                    lo_i, hi_i = int(lo), int(hi or lo)
                    if lo_i < 1 or hi_i < lo_i or hi_i > n_lines:
                        bad.append(f"{name}:{lineno}: {m.group(1)}:{part} outside its {n_lines} lines")
    assert count > 100, count
    assert not bad, "\n".join(bad)
