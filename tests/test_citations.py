"""Every reference citation (file.ts:N or file.ts:N-M) in this repository's sources and
documents points at lines that exist in the cited reference file, and a citation placed
beside a named reference function covers the line on which that function starts.

The reference's line counts and symbol lines are a committed fixture
(tests/golden/reference_lines.json, written by tests/golden/make_reference_lines.py), so
this check needs neither the reference checkout nor a GPU."""
import json
import os
import re

from webgpu_b200._build_paths import REPO_DIR

FIXTURE = json.load(open(os.path.join(REPO_DIR, "tests", "golden", "reference_lines.json")))
BY_NAME = {}
for rel, info in FIXTURE.items():
    BY_NAME.setdefault(os.path.basename(rel), []).append(info)
CITE = re.compile(r"([A-Za-z0-9_\-]+\.(?:ts|mjs)):(\d+(?:-\d+)?(?:,\d+(?:-\d+)?)*)")
# "Symbol (file.ts:ranges" or "Symbol, file.ts:ranges": the symbol should start inside the cited ranges
NAMED = re.compile(r"\b([A-Za-z_][A-Za-z0-9_]*),?\s*\(?`?(?:src/core/)?([A-Za-z0-9_\-]+\.ts):(\d+(?:-\d+)?(?:,\d+(?:-\d+)?)*)")
SKIP_DIRS = {".git", "_work", "gpurun_out", "_build", "__pycache__", ".pytest_cache", "baseline", "golden"}
# records written by the round driver and reviewer, not sources of this build
SKIP_FILES = {"SURVEY.md", "VERDICT.md", "ADVICE.md", "BASELINE.json"}
EXTS = (".py", ".c", ".cu", ".cuh", ".h", ".md")


def _files():
    for root, dirs, files in os.walk(REPO_DIR):
        dirs[:] = [d for d in dirs if d not in SKIP_DIRS]
        for f in files:
            if f.endswith(EXTS) and f not in SKIP_FILES and not f.startswith(("BENCH_", "SCALE_", "GPUTEST_")):
                yield os.path.join(root, f)


def _ranges(spec: str):
    for part in spec.split(","):
        a, _, b = part.partition("-")
        yield int(a), int(b or a)


def test_every_citation_is_inside_its_file():
    bad, seen = [], 0
    for path in _files():
        for i, line in enumerate(open(path, encoding="utf-8", errors="replace"), 1):
            for m in CITE.finditer(line):
                infos = BY_NAME.get(m.group(1))
                if not infos:
                    continue
                seen += 1
                n = max(info["lines"] for info in infos)
                for a, b in _ranges(m.group(2)):
                    if not (1 <= a <= b <= n):
                        bad.append(f"{os.path.relpath(path, REPO_DIR)}:{i}: {m.group(0)} (file has {n} lines)")
    assert seen > 100
    assert not bad, "\n".join(bad)


def test_named_citations_cover_the_symbol():
    bad, seen = [], 0
    for path in _files():
        for i, line in enumerate(open(path, encoding="utf-8", errors="replace"), 1):
            for m in NAMED.finditer(line):
                sym, fname = m.group(1), m.group(2)
                starts = [info["symbols"][sym] for info in BY_NAME.get(fname, []) if sym in info["symbols"]]
                if not starts:
                    continue
                seen += 1
                if not any(a <= s <= b for s in starts for a, b in _ranges(m.group(3))):
                    bad.append(f"{os.path.relpath(path, REPO_DIR)}:{i}: {sym} starts at line {starts[0]}, cited {m.group(0)}")
    assert seen >= 5
    assert not bad, "\n".join(bad)
