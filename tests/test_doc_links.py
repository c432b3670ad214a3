"""The product documents (docs/ and the readme) reference no missing file, and the checker finds
dead relative links and dead source paths in code spans (reference: scripts/check_doc_links.py)."""
from lake_b200.utils import doc_links


def test_product_documents_have_no_dead_references():
    files = doc_links.default_files()
    assert files
    assert doc_links.check(files) == []


def test_the_checker_finds_dead_links_and_paths(tmp_path):
    md = tmp_path / "x.md"
    (tmp_path / "there.md").write_text("ok")
    md.write_text("\n".join([
        "[fine](there.md#part) [web](https://example.com) [anchor](#top)",
        "[gone](missing.md)",
        "`csrc/host/tier/{tier,tier_bind}.cpp` `lake_b200/runtime/worker_engine.py:82-140` `pool/agents/native.py`",
        "`csrc/host/tier/{tier,nothere}.cpp` `not a/path.py` `x*.py` `torch.cuda.is_available()`",
    ]))
    dead = doc_links.check([str(md)])
    assert len(dead) == 2
    assert dead[0].endswith(":2: link missing.md") and dead[1].endswith(":4: path csrc/host/tier/nothere.cpp")
