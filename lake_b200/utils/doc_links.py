"""Dead-reference check for the repository's markdown documents.

Two kinds of reference are checked:

* relative markdown links (``[text](path#anchor)``), resolved against the document's folder
  (web links, mail links and bare anchors are skipped);
* code spans that name a repository file (``csrc/host/tier/tier.cpp``, ``pool/agents/native.py``,
  ``lake_b200/runtime/{worker,config}.py``), resolved against the repository root or the package
  folder; ``{a,b}`` alternatives are expanded, and spans with wildcards, spaces or a scheme are not
  paths and are skipped.

``python -m lake_b200.utils.doc_links [FILE ...]`` prints one line per dead reference and exits 1
if there is any (default: every markdown file under ``docs/`` and the top-level readme).

Reference parity: scripts/check_doc_links.py (relative links only); the code-span check is this
repository's addition, since its documents name source files in code spans.
"""
from __future__ import annotations

import glob
import itertools
import os
import re
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
PKG = os.path.join(ROOT, "lake_b200")
LINK = re.compile(r"\[[^\]]*\]\(([^)\s]+)[^)]*\)")
SPAN = re.compile(r"`([^`\n]+)`")
SKIP = ("http://", "https://", "mailto:", "#")
FILE_EXT = (".py", ".cpp", ".h", ".cu", ".cuh", ".md", ".sh", ".yaml", ".yml", ".proto", ".json", ".txt")


def _expand(span: str) -> list[str]:
    """`a/{b,c}.py` -> [a/b.py, a/c.py]."""
    parts = re.split(r"(\{[^{}]*\})", span)
    choices = [p[1:-1].split(",") if p.startswith("{") and p.endswith("}") else [p] for p in parts]
    return ["".join(c) for c in itertools.product(*choices)]


def _path_like(span: str) -> bool:
    if any(ch in span for ch in " *?<>$|=") or span.startswith(SKIP) or "://" in span:
        return False
    base = re.sub(r"\{[^{}]*\}", "x", span).split(":", 1)[0]  # file.py:12-30 names a file
    return "/" in base and base.endswith(FILE_EXT)


def _exists(path: str, md_dir: str) -> bool:
    path = path.split(":", 1)[0]
    return any(os.path.exists(os.path.join(base, path)) for base in (md_dir, ROOT, PKG))


def check(files: list[str]) -> list[str]:
    dead = []
    for md in files:
        md_dir = os.path.dirname(os.path.abspath(md))
        with open(md, encoding="utf-8") as f:
            for lineno, line in enumerate(f, 1):
                for target in LINK.findall(line):
                    if target.startswith(SKIP):
                        continue
                    path = target.split("#", 1)[0].split("?", 1)[0]
                    if path and not os.path.exists(os.path.join(md_dir, path)):
                        dead.append(f"{os.path.relpath(md, ROOT)}:{lineno}: link {target}")
                for span in SPAN.findall(line):
                    if not _path_like(span):
                        continue
                    for p in _expand(span):
                        if not _exists(p, md_dir):
                            dead.append(f"{os.path.relpath(md, ROOT)}:{lineno}: path {p}")
    return dead


def default_files() -> list[str]:
    return sorted(glob.glob(os.path.join(ROOT, "docs", "**", "*.md"), recursive=True)) + \
        sorted(glob.glob(os.path.join(ROOT, "README*.md")))


def main(argv: list[str] | None = None) -> int:
    files = (argv if argv else None) or default_files()
    dead = check(files)
    for d in dead:
        print("DEAD:", d)
    return 1 if dead else 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
