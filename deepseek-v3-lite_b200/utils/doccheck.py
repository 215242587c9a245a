"""Documentation checks: Markdown structure and code references.

Covers what the reference's docs tooling checks (``scripts/check_docs.py``
lint, ``tests/test_doc_refs.py`` doc-to-code resolution) for this tree's
Markdown files:

* structure: fenced code blocks are closed, heading levels never jump by
  more than one, relative links ``[text](path)`` point at existing files;
* code references: every backticked source path (``ops/engine.py``,
  ``csrc/gemm.cu``, ...) exists, searched relative to the document, the
  repository root and the package directory; a ``path.py:Name`` or
  ``path.py::Name`` reference also needs ``Name`` defined in that file
  (``def``, ``class`` or an assignment).

``python -m utils.doccheck FILE.md ...`` prints one line per problem and
exits non-zero if there is any.
"""
from __future__ import annotations

import re
import sys
from pathlib import Path
from typing import Iterable, List

PKG = Path(__file__).resolve().parent.parent
ROOT = PKG.parent
_SRC_EXT = r"(?:py|cu|cuh|cpp|h|yaml|yml|json|sh)"
_REF = re.compile(r"`([A-Za-z0-9_./-]+\." + _SRC_EXT + r")(?::{1,2}([A-Za-z_][A-Za-z0-9_.]*))?`")
_LINK = re.compile(r"\[[^\]]*\]\(([^)\s]+)\)")
_HEADING = re.compile(r"^(#{1,6})\s")


def _resolve(ref: str, doc: Path) -> Path | None:
    for base in (doc.parent, ROOT, PKG):
        p = (base / ref).resolve()
        if p.exists():
            return p
    return None


def _defines(path: Path, name: str) -> bool:
    leaf = name.split(".")[-1]
    text = path.read_text(encoding="utf-8", errors="replace")
    pat = re.compile(rf"^\s*(?:async\s+def|def|class)\s+{re.escape(leaf)}\b|^\s*{re.escape(leaf)}\s*[:=]"
                     rf"|\b{re.escape(leaf)}\s*\(", re.M)
    return bool(pat.search(text))


def check_file(doc: Path) -> List[str]:
    problems: List[str] = []
    lines = doc.read_text(encoding="utf-8").splitlines()
    fence, last_level = None, 0
    for n, line in enumerate(lines, 1):
        stripped = line.lstrip()
        if stripped.startswith("```") or stripped.startswith("~~~"):
            mark = stripped[:3]
            fence = None if fence == mark else (fence or mark)
            continue
        if fence:
            continue
        m = _HEADING.match(line)
        if m:
            level = len(m.group(1))
            if last_level and level > last_level + 1:
                problems.append(f"{doc}:{n}: heading jumps from level {last_level} to {level}")
            last_level = level
        for target in _LINK.findall(line):
            if re.match(r"^[a-z]+:", target) or target.startswith("#"):
                continue
            if _resolve(target.split("#")[0], doc) is None:
                problems.append(f"{doc}:{n}: link target not found: {target}")
        for ref, name in _REF.findall(line):
            if " " in ref or ref.startswith("/"):
                continue
            p = _resolve(ref, doc)
            if p is None:
                problems.append(f"{doc}:{n}: code reference not found: {ref}")
            elif name and not _defines(p, name):
                problems.append(f"{doc}:{n}: {name} not defined in {ref}")
    if fence:
        problems.append(f"{doc}: unclosed code fence")
    return problems


def check(paths: Iterable[str]) -> List[str]:
    out: List[str] = []
    for p in paths:
        out.extend(check_file(Path(p)))
    return out


def main(argv=None) -> int:
    problems = check(argv if argv is not None else sys.argv[1:])
    for p in problems:
        print(p)
    return 1 if problems else 0


if __name__ == "__main__":
    sys.exit(main())
