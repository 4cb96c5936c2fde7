"""Writes tests/golden/reference_lines.json: the line count of every Python, Markdown and TOML file of the reference
checkout (rkinas/basal 2.8.1), so that tests/test_citations.py can check the `file.py:N` citations of this repository
on a machine without the checkout.

    python tests/golden/make_reference_index.py <reference checkout>
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def index(root):
    out = {}
    for d, dirs, files in os.walk(root):
        dirs[:] = sorted(x for x in dirs if not x.startswith("."))
        for f in sorted(files):
            if f.endswith((".py", ".md", ".toml")):
                p = os.path.join(d, f)
                with open(p, "rb") as fh:
                    out[os.path.relpath(p, root)] = fh.read().count(b"\n")
    return out


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    with open(os.path.join(HERE, "reference_lines.json"), "w") as fh:
        json.dump(index(sys.argv[1]), fh, indent=0, sort_keys=True)
        fh.write("\n")
