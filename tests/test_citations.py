"""Every `file.py:N` citation of the reference in this repository's code and documents points at a line that exists
in that file of the reference (rkinas/basal 2.8.1), checked against tests/golden/reference_lines.json (each reference
file's line count, written by tests/golden/make_reference_index.py). A bare file name resolves to basal/<name>, then
tests/<name>; continuation spans (`, :40-45`) belong to the file named before them. No GPU."""
import json
import os
import re

from conftest import GOLDEN, ROOT

CHECKED = ("basal_b200", "include", "oracle", "tests", "profiles")
TOP = ("bench.py", "__graft_entry__.py", "DESIGN.md", "INTEGRATION.md", "README.md")
SUFFIXES = (".py", ".h", ".cu", ".cuh", ".md", ".txt")
CITE = re.compile(r"((?:[\w.-]+/)*[\w-]+\.(?:py|md|toml))((?::\d+(?:-\d+)?)(?:(?:,\s*|\s+and\s+)(?::\d+(?:-\d+)?))*)")


def _files():
    for f in TOP:
        yield os.path.join(ROOT, f)
    for d in CHECKED:
        for base, dirs, files in os.walk(os.path.join(ROOT, d)):
            dirs[:] = [x for x in dirs if not x.startswith((".", "__"))]
            for f in files:
                if f.endswith(SUFFIXES):
                    yield os.path.join(base, f)


def _resolve(name, lines):
    if "/" in name:
        hits = [p for p in lines if p == name or p.endswith("/" + name)]
    else:
        hits = [p for p in (f"basal/{name}", f"tests/{name}") if p in lines]
    return hits[0] if hits else None


def test_every_reference_citation_points_at_an_existing_line():
    with open(os.path.join(GOLDEN, "reference_lines.json")) as fh:
        lines = json.load(fh)
    checked, bad = 0, []
    for path in _files():
        with open(path, errors="replace") as fh:
            text = fh.read()
        for ln, line in enumerate(text.splitlines(), 1):
            for m in CITE.finditer(line):
                target = _resolve(m.group(1), lines)
                if target is None:
                    continue  # a file of this repository, not of the reference
                for a, b in re.findall(r":(\d+)(?:-(\d+))?", m.group(2)):
                    lo, hi = int(a), int(b or a)
                    checked += 1
                    if not 1 <= lo <= hi <= lines[target]:
                        bad.append(f"{os.path.relpath(path, ROOT)}:{ln}: {m.group(0)} ({target} has "
                                   f"{lines[target]} lines)")
    assert checked > 100, checked
    assert not bad, "\n".join(bad)
