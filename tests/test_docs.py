"""Documentation checks (CPU): the user-facing Markdown files resolve every
code reference and link, and the checker catches broken ones."""
from pathlib import Path

from utils import doccheck

ROOT = Path(__file__).resolve().parent.parent


def test_user_docs_resolve():
    docs = [ROOT / "README.md"] + sorted((ROOT / "profiles").glob("*.md"))
    assert doccheck.check(str(p) for p in docs) == []


def test_checker_reports_problems(tmp_path):
    doc = tmp_path / "bad.md"
    doc.write_text("# Title\n\n### Skipped a level\n\nSee `ops/not_a_file.py` and `ops/engine.py:NoSuchName`.\n"
                   "[link](missing.md)\n\n```\nunclosed\n")
    problems = doccheck.check([str(doc)])
    kinds = " ".join(problems)
    assert "heading jumps" in kinds and "not_a_file.py" in kinds and "NoSuchName" in kinds
    assert "missing.md" in kinds and "unclosed code fence" in kinds
    assert doccheck.check_file(tmp_path / "bad.md") == problems
